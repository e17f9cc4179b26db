// Device-side remap (R2 / R3 / R6) shared by the standalone remap kernel and the fused decode
// front kernel.  See remap.cu for the reference rules and the parallel formulation.
#pragma once

#include "common.cuh"

namespace nvmoe {


constexpr int kMaxExpertsRemap = 16384;
constexpr int kMaxSlotsRemap = 4096;

struct RemapParams {
    nvmoe_slot_table t;
    const int32_t* ids;
    int64_t ids_stride;  // bytes
    int32_t* out;
    int64_t out_stride;  // bytes
    int top_k;
    int n_tok;
    int is_decode;
    nvmoe_miss_list m;
};

__device__ __forceinline__ const int32_t* id_ptr(const int32_t* base, int64_t stride, int k,
                                                 int p) {
    const int row = p / k, col = p - row * k;
    return reinterpret_cast<const int32_t*>(reinterpret_cast<const char*>(base) + row * stride) +
           col;
}

// Ordered stream compaction of positions [0, n) with predicate pred(p): calls emit(p, rank)
// in every thread for each selected p, rank = number of selected positions before p.
template <typename Pred, typename Emit>
__device__ inline int ordered_compact(int n, int* warp_sums, Pred pred, Emit emit) {
    int running = 0;
    for (int base = 0; base < n; base += blockDim.x) {
        const int p = base + threadIdx.x;
        const int f = (p < n && pred(p)) ? 1 : 0;
        int total;
        const int ex = block_exclusive_scan(f, warp_sums, &total);
        if (f) emit(p, running + ex);
        running += total;
    }
    return running;
}


__host__ __device__ inline size_t remap_smem_bytes(int n_expert, int cache_size) {
    int s2 = 1;
    while (s2 < cache_size) s2 <<= 1;
    return (size_t)s2 * 8 + (size_t)n_expert * 4 * 3 + (size_t)cache_size * 4;
}

// Whole remap call by one thread block (any multiple of 32 threads).  smem_raw: remap_smem_bytes.
// Returns the call's status (the same value in every thread).
__device__ inline int remap_block(const RemapParams& P, unsigned char* smem_raw) {
    const int E = P.t.n_expert;
    const int S = P.t.cache_size;
    int S2 = 1;
    while (S2 < S) S2 <<= 1;
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem_raw);  // [S2]
    int* first_pos = reinterpret_cast<int*>(keys + S2);                          // [E]
    int* uniq = first_pos + E;                                                   // [E]
    int* active = uniq + E;                                                      // [S]
    int* miss_r = active + S;                                                    // [E]
    __shared__ int warp_sums[33];
    __shared__ int s_err, s_nuniq, s_nmiss;
    __syncthreads();  // smem_raw may be reused from an earlier phase of the caller

    const int n = P.n_tok * P.top_k;
    const int tid = threadIdx.x;
    if (tid == 0) s_err = NVMOE_OK;
    for (int i = tid; i < E; i += blockDim.x) first_pos[i] = 0x7fffffff;
    for (int i = tid; i < S; i += blockDim.x) active[i] = 0;
    __syncthreads();

    // 1. validate ids and record the first position of each distinct id
    for (int p = tid; p < n; p += blockDim.x) {
        const int id = *id_ptr(P.ids, P.ids_stride, P.top_k, p);
        if (id < 0 || id >= E) {
            atomicExch(&s_err, NVMOE_ERR_BAD_EXPERT_ID);
        } else {
            atomicMin(&first_pos[id], p);
        }
    }
    __syncthreads();
    if (s_err != NVMOE_OK) {
        if (tid == 0) {
            P.m.counts[0] = 0;
            P.m.counts[1] = 0;
            P.m.counts[2] = s_err;
            P.m.counts[3] = n;
        }
        return NVMOE_ERR_BAD_EXPERT_ID;
    }

    // 2. distinct ids in first-occurrence order
    const int nuniq = ordered_compact(
        n, warp_sums,
        [&](int p) { return first_pos[*id_ptr(P.ids, P.ids_stride, P.top_k, p)] == p; },
        [&](int p, int r) { uniq[r] = *id_ptr(P.ids, P.ids_stride, P.top_k, p); });
    __syncthreads();
    if (nuniq > S) {
        if (tid == 0) {
            P.m.counts[0] = nuniq;
            P.m.counts[1] = 0;
            P.m.counts[2] = NVMOE_ERR_CACHE_OVERFLOW;
            P.m.counts[3] = n;
        }
        return NVMOE_ERR_CACHE_OVERFLOW;
    }

    // 3. hits / misses; hits mark their slot active
    const int id_base = P.t.id_base;
    for (int r = tid; r < nuniq; r += blockDim.x) {
        const int s = P.t.slot_of_real[id_base + uniq[r]];
        if (s >= 0 && s < S) active[s] = 1;
    }
    __syncthreads();
    const int nmiss = ordered_compact(
        nuniq, warp_sums,
        [&](int r) {
            const int s = P.t.slot_of_real[id_base + uniq[r]];
            return !(s >= 0 && s < S);
        },
        [&](int r, int j) { miss_r[j] = r; });
    if (tid == 0) {
        s_nuniq = nuniq;
        s_nmiss = nmiss;
    }
    const uint32_t step = *P.t.current_step + 1u;

    // 4. victim order: bitonic sort of the candidate keys (skipped when everything hit)
    if (nmiss > 0) {
        const int start = (P.is_decode && P.t.pinned_k > 0) ? min(P.t.pinned_k, S) : 0;
        for (int s = tid; s < S2; s += blockDim.x) {
            unsigned long long k = ~0ull;
            if (s < S && !active[s]) {
                const int occ = P.t.real_in_slot[s];
                const bool hi = s >= start;
                const unsigned long long cls = occ < 0 ? (hi ? 0ull : 2ull) : (hi ? 1ull : 3ull);
                const unsigned long long lu = occ < 0 ? 0ull : (unsigned long long)P.t.slot_last_used[s];
                k = (cls << 62) | (lu << 24) | (unsigned long long)s;
            }
            keys[s] = k;
        }
        __syncthreads();
        for (int size = 2; size <= S2; size <<= 1) {
            for (int stride = size >> 1; stride > 0; stride >>= 1) {
                for (int i = tid; i < (S2 >> 1); i += blockDim.x) {
                    const int lo = 2 * i - (i & (stride - 1));
                    const int hi = lo + stride;
                    const bool up = ((lo & size) == 0);
                    const unsigned long long a = keys[lo], b = keys[hi];
                    if ((a > b) == up) {
                        keys[lo] = b;
                        keys[hi] = a;
                    }
                }
                __syncthreads();
            }
        }
        // 5. install misses (distinct slots, distinct evicted ids: no write conflicts)
        for (int j = tid; j < nmiss; j += blockDim.x) {
            const int r = miss_r[j];
            const int e = uniq[r];
            const int s = (int)(keys[j] & 0xffffffull);
            const int ev = P.t.real_in_slot[s];
            if (ev >= 0) P.t.slot_of_real[ev] = -1;
            P.t.real_in_slot[s] = id_base + e;
            P.t.slot_of_real[id_base + e] = s;
            P.t.slot_last_used[s] = step;
            P.m.miss_ids[j] = e;
            P.m.miss_slots[j] = s;
            P.m.evicted_ids[j] = ev;
        }
    }
    __syncthreads();
    // hits: stamp; every distinct id: report
    for (int r = tid; r < nuniq; r += blockDim.x) {
        const int e = uniq[r];
        const int s = P.t.slot_of_real[id_base + e];
        P.m.unique_ids[r] = e;
        P.m.unique_slot[r] = s;
        P.t.slot_last_used[s] = step;
    }
    // the hit flags need the pre-call state: a miss index list is in miss_r
    for (int r = tid; r < nuniq; r += blockDim.x) P.m.unique_hit[r] = 1;
    __syncthreads();
    for (int j = tid; j < nmiss; j += blockDim.x) P.m.unique_hit[miss_r[j]] = 0;

    // 6. rewrite ids -> slots (same thread reads then writes position p: in-place safe)
    for (int p = tid; p < n; p += blockDim.x) {
        const int id = *id_ptr(P.ids, P.ids_stride, P.top_k, p);
        const int s = P.t.slot_of_real[id_base + id];
        *const_cast<int32_t*>(id_ptr(P.out, P.out_stride, P.top_k, p)) = s;
    }
    if (tid == 0) {
        *P.t.current_step = step;
        P.m.counts[0] = s_nuniq;
        P.m.counts[1] = s_nmiss;
        P.m.counts[2] = NVMOE_OK;
        P.m.counts[3] = n;
    }
    __syncthreads();
    return NVMOE_OK;
}

}  // namespace nvmoe
