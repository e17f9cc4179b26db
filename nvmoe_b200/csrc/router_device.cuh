// R1 router top-k, warp-level device function shared by the router kernel and the fused decode
// front kernel (see router.cu for the reference behaviour).
#pragma once

#include "common.cuh"

namespace nvmoe {

constexpr int kMaxExperts = 1024;
constexpr int kMaxTopK = 32;

// Order-preserving map of a selection key to uint32: a larger float gives a larger integer, -0
// maps like +0 (they compare equal), and -inf maps to 0x007FFFFF, so 0 is free to mean "no
// candidate" (experts past n_expert and experts already picked).
__device__ __forceinline__ uint32_t ordered_key(float k) {
    const uint32_t u = __float_as_uint(k == 0.f ? 0.f : k);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// Arg-max of a lane's key tile: the largest key (max tree) and the lowest tile index holding it
// (equality bit mask + find-first-set; index arrays in the tree would double the registers).
template <int PL>
__device__ __forceinline__ void tile_argmax(const uint32_t (&key)[PL], uint32_t& m, int& mi) {
    uint32_t t[PL / 2 > 0 ? PL / 2 : 1];
    if constexpr (PL == 1) {
        t[0] = key[0];
    } else {
#pragma unroll
        for (int i = 0; i < PL / 2; ++i) t[i] = max(key[i], key[i + PL / 2]);
#pragma unroll
        for (int w = PL / 4; w >= 1; w /= 2)
#pragma unroll
            for (int i = 0; i < w; ++i) t[i] = max(t[i], t[i + w]);
    }
    m = t[0];
    uint32_t eq = 0;
#pragma unroll
    for (int i = 0; i < PL; ++i) eq |= (key[i] == m ? 1u : 0u) << i;
    mi = __ffs(eq) - 1;
}

// The k largest keys of a warp's key tile (expert e = 32 i + lane in key[i] of lane e % 32; 0 =
// no candidate), ties to the smallest e: a warp max of the lanes' tile maxima (redux.sync), then
// a warp min over the ids of the lanes that hold that key (each lane's arg-max already prefers
// its lowest id).  Only the winning lane clears its key and recomputes its arg-max.  The key
// order is a strict total order, so the result does not depend on scheduling.  Lane j < k gets
// pick j: its e and key.
template <int PL>
__device__ __forceinline__ void tile_pick(uint32_t (&key)[PL], int k, int& my_e,
                                          uint32_t& my_key) {
    const int lane = threadIdx.x & 31;
    uint32_t lm;
    int li;
    tile_argmax<PL>(key, lm, li);
    for (int j = 0; j < k; ++j) {
        const uint32_t m = __reduce_max_sync(0xffffffffu, lm);
        const uint32_t cand = (lm == m) ? (uint32_t)(li * 32 + lane) : 0xffffffffu;
        const uint32_t e = __reduce_min_sync(0xffffffffu, cand);
        if (lane == j) my_e = (int)e, my_key = m;
        if ((int)(e & 31) == lane) {
            // clear with a compare per element (an indexed store would put the tile in local
            // memory), then the new arg-max of this lane
#pragma unroll
            for (int i = 0; i < PL; ++i) key[i] = (i == li) ? 0u : key[i];
            tile_argmax<PL>(key, lm, li);
        }
    }
}

// The same picks as tile_pick, by threshold: T = the k-th largest of the 32 lanes' tile maxima
// is a lower bound of the k-th largest key of the row (those k maxima are k distinct keys), so
// the k picks are among the keys >= T.  The candidates (usually k to 2k of them) are gathered in
// shared memory as (key, ~e) pairs and sorted in one bitonic pass across the warp, which orders
// equal keys by ascending e as the pick loop does.  Returns false (nothing written) when there
// are more than 32 candidates or fewer than k keys; the caller then runs tile_pick.  Uniform
// across the warp; key is not modified.
__device__ __forceinline__ unsigned long long* topk_candidate_buffer() {
    __shared__ unsigned long long buf[32][32];  // one 32-entry buffer per warp of the block
    return buf[threadIdx.x >> 5];
}

template <int PL>
__device__ __forceinline__ bool tile_pick_threshold(const uint32_t (&key)[PL], int k, int& my_e,
                                                    uint32_t& my_key) {
    const int lane = threadIdx.x & 31;
    uint32_t v = 0;
#pragma unroll
    for (int i = 0; i < PL; ++i) v = max(v, key[i]);
    // bitonic sort of the lane maxima, descending across the warp
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
        const bool desc = (lane & size) == 0;
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const uint32_t o = __shfl_xor_sync(0xffffffffu, v, j);
            v = (((lane & j) == 0) == desc) ? max(v, o) : min(v, o);
        }
    }
    const uint32_t T = __shfl_sync(0xffffffffu, v, k - 1);
    uint32_t m = 0;
#pragma unroll
    for (int i = 0; i < PL; ++i) m |= (key[i] >= T ? 1u : 0u) << i;
    if (T == 0u) m = 0;
    const int c = __popc(m);
    const int C = (int)__reduce_add_sync(0xffffffffu, (unsigned)c);
    if (T == 0u || C > 32) return false;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int n = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += n;
    }
    unsigned long long* buf = topk_candidate_buffer();
    int pos = inc - c;
#pragma unroll
    for (int i = 0; i < PL; ++i)
        if ((m >> i) & 1u)
            buf[pos++] = ((unsigned long long)key[i] << 32) | (0xffffffffu - (uint32_t)(i * 32 + lane));
    __syncwarp();
    unsigned long long x = lane < C ? buf[lane] : 0ull;
    __syncwarp();
#pragma unroll
    for (int size = 2; size <= 32; size <<= 1) {
        const bool desc = (lane & size) == 0;
#pragma unroll
        for (int j = size >> 1; j > 0; j >>= 1) {
            const unsigned long long o = __shfl_xor_sync(0xffffffffu, x, j);
            x = (((lane & j) == 0) == desc) ? (x > o ? x : o) : (x < o ? x : o);
        }
    }
    if (lane < k) {
        my_key = (uint32_t)(x >> 32);
        my_e = (int)(0xffffffffu - (uint32_t)x);
    }
    return true;
}

// Selection keys of n experts (the row's first n) into a PL-per-lane tile, then the top k.
template <int PL>
__device__ __forceinline__ void row_select(const float* __restrict__ lr, int n, int k, int mode,
                                           const float* __restrict__ bias, int& my_id,
                                           uint32_t& my_key) {
    const int lane = threadIdx.x & 31;
    const uint32_t kNanKey = 0x007FFFFFu;  // ordered_key(-inf): NaN keys never win
    // all loads first (clamped in-row addresses), so they are in flight together
    uint32_t key[PL];
#pragma unroll
    for (int i = 0; i < PL; ++i) key[i] = __float_as_uint(__ldcg(lr + min(i * 32 + lane, n - 1)));
    if (mode != NVMOE_ROUTER_SOFTMAX) {
        // sigmoid score plus the selection bias
#pragma unroll
        for (int i = 0; i < PL; ++i) {
            const float b = bias ? __ldcg(bias + min(i * 32 + lane, n - 1)) : 0.0f;
            key[i] = __float_as_uint(1.0f / (1.0f + expf(-__uint_as_float(key[i]))) + b);
        }
    }
#pragma unroll
    for (int i = 0; i < PL; ++i) {
        // softmax is monotone: select on the logits themselves
        const float c = __uint_as_float(key[i]);
        key[i] = (i * 32 + lane >= n) ? 0u : ((c != c) ? kNanKey : ordered_key(c));
    }
    if (!tile_pick_threshold<PL>(key, k, my_id, my_key)) tile_pick<PL>(key, k, my_id, my_key);
}

// Top-k of one token row by one warp; writes ids / weights [top_k] (called by all 32 lanes).
// Rows of up to 512 experts are one register tile; longer rows (up to kMaxExperts) select the
// top k of each 512-expert half and merge the two lists with a 2-per-lane tile: its proxy order
// (half, pick) equals the expert-id order among equal keys, because half 0 holds the lower ids
// and each half's picks of equal key come in ascending id.
__device__ __forceinline__ void router_topk_warp(const float* __restrict__ lr, int n_expert,
                                                 int top_k, int mode,
                                                 const float* __restrict__ bias, int norm_topk,
                                                 float scaling, int32_t* __restrict__ ids_row,
                                                 float* __restrict__ w_row) {
    const int lane = threadIdx.x & 31;
    int my_id = -1;
    uint32_t my_key = 0;
    if (n_expert <= 64) {
        row_select<2>(lr, n_expert, top_k, mode, bias, my_id, my_key);
    } else if (n_expert <= 128) {
        row_select<4>(lr, n_expert, top_k, mode, bias, my_id, my_key);
    } else if (n_expert <= 256) {
        row_select<8>(lr, n_expert, top_k, mode, bias, my_id, my_key);
    } else if (n_expert <= 512) {
        row_select<16>(lr, n_expert, top_k, mode, bias, my_id, my_key);
    } else {
        const int n1 = n_expert - 512, k1 = min(top_k, n1);
        int id0 = -1, id1 = -1;
        uint32_t key0 = 0, key1 = 0;
        row_select<16>(lr, 512, top_k, mode, bias, id0, key0);
        row_select<16>(lr + 512, n1, k1, mode, bias ? bias + 512 : nullptr, id1, key1);
        uint32_t key2[2] = {lane < top_k ? key0 : 0u, lane < k1 ? key1 : 0u};
        int pe = -1;
        tile_pick<2>(key2, top_k, pe, my_key);
        const int pl = pe & 31;
        const int a = __shfl_sync(0xffffffffu, id0, pl), b = __shfl_sync(0xffffffffu, id1, pl);
        my_id = (pe >> 5) ? 512 + b : a;
    }

    // the picked values: softmax the logit (its key maps back to it, except the NaN / -inf
    // key, which is re-read), sigmoid the plain score (re-read)
    const bool mine = lane < top_k;
    float my_val = 0.f;
    if (mine) {
        if (mode == NVMOE_ROUTER_SOFTMAX && my_key != 0x007FFFFFu) {
            my_val = __uint_as_float((my_key & 0x80000000u) ? (my_key & 0x7fffffffu) : ~my_key);
        } else {
            const float l = __ldcg(lr + my_id);
            my_val = (mode == NVMOE_ROUTER_SOFTMAX) ? l : 1.0f / (1.0f + expf(-l));
        }
    }
    const float first_val = __shfl_sync(0xffffffffu, my_val, 0);

    // Full-softmax denominator (only when the top-k weights are not renormalised): per-lane
    // sums over e = lane, lane + 32, ... then a butterfly.
    float full_denom = 0.f;
    if (mode == NVMOE_ROUTER_SOFTMAX && !norm_topk) {
        for (int e = lane; e < n_expert; e += 32) {
            const float l = __ldcg(lr + e);
            if (l == l) full_denom += expf(l - first_val);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) full_denom += __shfl_xor_sync(0xffffffffu, full_denom, o);
    }

    float w;
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        // probabilities relative to the row maximum (= the first pick)
        w = mine ? expf(my_val - first_val) : 0.f;
    } else {
        w = mine ? my_val : 0.f;
    }
    // sum of the picks in pick order (lane 0 first), identical on every lane (a loop: this code
    // runs once per row, cold in the instruction cache, where fetching an unrolled copy costs
    // more than the loop)
    float sum = 0.f;
#pragma unroll 1
    for (int j = 0; j < top_k; ++j) sum += __shfl_sync(0xffffffffu, w, j);
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        const float denom = norm_topk ? sum : full_denom;
        w = w / denom * scaling;
    } else {
        w = (norm_topk ? w / (sum + 1e-20f) : w) * scaling;
    }
    if (mine) {
        ids_row[lane] = my_id;
        w_row[lane] = w;
    }
}

}  // namespace nvmoe
