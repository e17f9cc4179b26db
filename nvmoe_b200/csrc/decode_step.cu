// One decode layer step (engine path): fused router + remap + FFN grouping kernel, then the
// optional refill gather and the FFN kernels, all chained with programmatic dependent launch.
//
// The front kernel is one CTA: warps compute the top-k of the token rows (router_device.cuh)
// while the slot tables stream into shared memory, then the block runs the remap and the FFN
// grouping entirely in shared memory and stores the results.  Replaces three launches (router,
// remap, FFN prep) and their dependent global-memory round trips on the latency-critical
// small-batch decode path.
#include "common.cuh"
#include "ffn_common.cuh"
#include "remap_device.cuh"
#include "router_device.cuh"

#include <algorithm>

extern "C" int nvmoe_refill_gather(const nvmoe_refill_bank* banks, int n_banks,
                                   const nvmoe_miss_list* misses, const int32_t* host_slot_of_id,
                                   int32_t n_gpu_slots, nvmoe_stream_t stream);

namespace nvmoe {
namespace {

constexpr int kFrontThreads = 512;  // at most 16 warps; 128 registers per thread for the top-k tile
constexpr int kFrontMaxIds = 8192;  // routed (token, k) entries per call on this path
constexpr int kFrontMaxSlots = 1024;

struct FrontParams {
    const float* logits;
    int64_t lstride;
    int mode;
    const float* bias;
    int norm_topk;
    float scaling;
    RemapParams rp;  // rp.out: slot ids [n_tok, k] (global), rp.ids unused
    float* weights;
    FfnParams fp;
    int early;  // the workspace and miss list are not the previous step's: written before the wait
    int inputs_after_wait;  // the logits / token rows come from the kernel before this one
    const int32_t* rids;    // logits == NULL: routed expert ids [n_tok, K] (< 0: empty entry)
    const float* rw;        //                 and their combine weights [n_tok, K]
    int64_t rstride;        //                 elements between their rows
};

__device__ __forceinline__ void cp_async4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
    asm volatile("cp.async.commit_group;\n\tcp.async.wait_group 0;" ::: "memory");
}

// Shared-memory layout of the front kernel (ints unless noted).
struct FrontSmem {
    int sor, ris, lu, first, uniq, uslot, miss_r, act, cnt, gbase, aidx, sids, sw, pe, ent_tok,
        ent_w, keys, total;
};
__host__ __device__ inline FrontSmem front_smem(int E, int S, int n, int n_ent) {
    int s2 = 1;
    while (s2 < S) s2 <<= 1;
    FrontSmem L;
    int o = 0;
    L.keys = o;  // u64 [s2]
    o += 8 * s2;
    L.sor = o;
    o += 4 * E;
    L.ris = o;
    o += 4 * S;
    L.lu = o;
    o += 4 * S;
    L.first = o;
    o += 4 * E;
    L.uniq = o;
    o += 4 * E;
    L.uslot = o;
    o += 4 * E;
    L.miss_r = o;
    o += 4 * E;
    L.act = o;
    o += 4 * S;
    L.cnt = o;
    o += 4 * S;
    L.gbase = o;
    o += 4 * S;
    L.aidx = o;
    o += 4 * S;
    L.sids = o;
    o += 4 * n;
    L.sw = o;
    o += 4 * n;
    L.pe = o;
    o += 4 * n;
    L.ent_tok = o;
    o += 4 * n_ent;
    L.ent_w = o;
    o += 4 * n_ent;
    L.total = o;
    return L;
}

// Token rows -> f16 and the shared-expert gate, one warp per token (no block barrier).  The
// row's loads are issued in batches of 8 x 16 bytes per lane before any of them is used; the
// conversion is packed (two values per instruction) and each mode has its own loop, so little
// code runs: this kernel's code is cold in the instruction cache at every launch.
__device__ __forceinline__ __half2 bf16x2_to_half2(uint32_t v) {
    return __floats2half2_rn(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}

__device__ __forceinline__ void front_convert_token(const FfnParams& P, int t, int lane) {
    const int H = P.pool.hidden;
    const uint16_t* xr = P.x + (int64_t)t * P.x_stride;
    __half* x16 = wsp<__half>(P, P.L.x16) + (int64_t)t * H;
    constexpr int kBatch = 8;
    if (!P.use_fp4) {
        for (int i0 = lane * 8; i0 < H; i0 += 256 * kBatch) {
            uint4 v[kBatch];
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int i = i0 + b * 256;
                v[b] = i < H ? *reinterpret_cast<const uint4*>(xr + i) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int b = 0; b < kBatch; ++b) {
                const int i = i0 + b * 256;
                if (i >= H) break;
                __half2 o[4] = {bf16x2_to_half2(v[b].x), bf16x2_to_half2(v[b].y),
                                bf16x2_to_half2(v[b].z), bf16x2_to_half2(v[b].w)};
                *reinterpret_cast<uint4*>(x16 + i) = *reinterpret_cast<const uint4*>(o);
            }
        }
    } else {  // the row's FP4 term exponent
        float amax = 0.f;
#pragma unroll 1
        for (int i = lane * 2; i < H; i += 64) {
            const uint32_t v = *reinterpret_cast<const uint32_t*>(xr + i);
            amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(v << 16)),
                                     fabsf(__uint_as_float(v & 0xffff0000u))));
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        if (lane == 0) wsp<int>(P, P.L.xk)[t] = fp4_row_exp(amax);
    }
    if (P.shared_gate) {
        float dot = 0.f;
#pragma unroll 1
        for (int i = lane * 2; i < H; i += 64) {
            const uint32_t v = *reinterpret_cast<const uint32_t*>(xr + i);
            const uint32_t g = *reinterpret_cast<const uint32_t*>(P.shared_gate + i);
            dot = fmaf(__uint_as_float(v << 16), __uint_as_float(g << 16), dot);
            dot = fmaf(__uint_as_float(v & 0xffff0000u), __uint_as_float(g & 0xffff0000u), dot);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if (lane == 0) wsp<float>(P, P.L.sg)[t] = 1.0f / (1.0f + expf(-dot));
    }
}

// Router top-k -> slot remap -> FFN grouping for one decode step, in one CTA.  Every table the
// step needs is prefetched into shared memory with cp.async while the warps load their logit
// rows and token rows, so global memory costs one round trip; results are stored at the end.
// Same rules as remap_device.cuh / ffn_common.cuh (eval_cb, moe_cache_probe.cpp:627-753,955-970).
__global__ void __launch_bounds__(kFrontThreads, 1) decode_front_kernel(FrontParams F) {
    extern __shared__ __align__(16) unsigned char smem[];
    __shared__ int warp_sums[33];
    __shared__ unsigned long long warp_sums64[33];
    __shared__ int s_err, s_step;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nthr = blockDim.x, nw = nthr >> 5;
    const int E = F.rp.t.n_expert, S = F.rp.t.cache_size, K = F.rp.top_k, n_tok = F.rp.n_tok;
    const int n = n_tok * K;
    const int id_base = F.rp.t.id_base;
    const FfnParams& P = F.fp;
    const FrontSmem L = front_smem(E, S, n, n + n_tok);
    unsigned long long* keys = reinterpret_cast<unsigned long long*>(smem + L.keys);
    int* sor = reinterpret_cast<int*>(smem + L.sor);
    int* ris = reinterpret_cast<int*>(smem + L.ris);
    uint32_t* lu = reinterpret_cast<uint32_t*>(smem + L.lu);
    int* first = reinterpret_cast<int*>(smem + L.first);
    int* uniq = reinterpret_cast<int*>(smem + L.uniq);
    int* uslot = reinterpret_cast<int*>(smem + L.uslot);
    int* miss_r = reinterpret_cast<int*>(smem + L.miss_r);
    int* act = reinterpret_cast<int*>(smem + L.act);
    int* cnt = reinterpret_cast<int*>(smem + L.cnt);
    int* gbase = reinterpret_cast<int*>(smem + L.gbase);
    int* sids = reinterpret_cast<int*>(smem + L.sids);
    float* sw = reinterpret_cast<float*>(smem + L.sw);
    int* ent_tok_s = reinterpret_cast<int*>(smem + L.ent_tok);
    float* ent_w_s = reinterpret_cast<float*>(smem + L.ent_w);
    int* aidx = reinterpret_cast<int*>(smem + L.aidx);
    int* pe = reinterpret_cast<int*>(smem + L.pe);

    // Everything but the buffers shared with the kernel before this one runs before the
    // dependency wait, while that kernel (normally the previous layer's FFN, which leaves an SM
    // free for this CTA) is still running: routing, the remap with this layer's table, slot-id
    // and weight writes, and the grouping in shared memory.  The router logits must be complete
    // when the previous kernel triggers its dependents.  After the wait: the miss list (the FFN
    // before this kernel may read the same one while copying its own misses in), the token rows
    // and the FFN workspace; with early outputs (the caller alternates two sets of these
    // buffers) those too come before the wait, and the token rows must then also be complete
    // when the previous kernel triggers.
    grid_dep_launch();
    // ---- A. one round trip: table prefetch (async) while the warps route their tokens
    for (int e = tid; e < E; e += nthr) cp_async4(sor + e, F.rp.t.slot_of_real + id_base + e);
    for (int s = tid; s < S; s += nthr) {
        cp_async4(ris + s, F.rp.t.real_in_slot + s);
        cp_async4(lu + s, F.rp.t.slot_last_used + s);
        act[s] = 0;
        cnt[s] = 0;
    }
    for (int e = tid; e < E; e += nthr) first[e] = 0x7fffffff;
    if (tid == 0) {
        s_err = NVMOE_OK;
        s_step = (int)(*F.rp.t.current_step + 1u);
    }
    // in a stack whose layers depend on each other the logits are the router gate's output;
    // pre-routed ids / weights (no logits) always come from the launches before this one
    if (F.inputs_after_wait || !F.logits) grid_dep_wait();
    if (F.logits) {
        for (int t = warp; t < n_tok; t += nw)
            router_topk_warp(F.logits + (int64_t)t * F.lstride, E, K, F.mode, F.bias,
                             F.norm_topk, F.scaling, sids + t * K, sw + t * K);
    } else {
        for (int p = tid; p < n; p += nthr) {
            const int64_t o = (int64_t)(p / K) * F.rstride + p % K;
            sids[p] = __ldcg(F.rids + o);
            sw[p] = __ldcg(F.rw + o);
        }
    }
    cp_async_wait_all();
    __syncthreads();

    // ---- B. remap in shared memory; this layer's tables and the miss list are written here
    for (int p = tid; p < n; p += nthr) {
        const int id = sids[p];  // a negative id is an empty entry (pre-routed calls)
        if (id >= E)
            s_err = NVMOE_ERR_BAD_EXPERT_ID;
        else if (id >= 0)
            atomicMin(&first[id], p);
    }
    __syncthreads();
    int status = s_err;
    int nuniq = 0, nmiss = 0;
    const uint32_t step = (uint32_t)s_step;
    if (status == NVMOE_OK) {
        nuniq = ordered_compact(n, warp_sums,
                                [&](int p) { return sids[p] >= 0 && first[sids[p]] == p; },
                                [&](int p, int r) { uniq[r] = sids[p]; });
        __syncthreads();
        if (nuniq > S) status = NVMOE_ERR_CACHE_OVERFLOW;
    }
    if (status == NVMOE_OK) {
        for (int r = tid; r < nuniq; r += nthr) {
            const int e = uniq[r];
            first[e] = r;  // id -> rank from here on
            const int s = sor[e];
            const bool hit = s >= 0 && s < S;
            uslot[r] = hit ? s : -1;
            if (hit) act[s] = 1;
        }
        __syncthreads();
        nmiss = ordered_compact(nuniq, warp_sums, [&](int r) { return uslot[r] < 0; },
                                [&](int r, int j) { miss_r[j] = r; });
        __syncthreads();
        if (nmiss > 0) {
            int S2 = 1;
            while (S2 < S) S2 <<= 1;
            const int start = (F.rp.is_decode && F.rp.t.pinned_k > 0) ? min(F.rp.t.pinned_k, S) : 0;
            for (int s = tid; s < S2; s += nthr) {
                unsigned long long k = ~0ull;
                if (s < S && !act[s]) {
                    const int occ = ris[s];
                    const bool hi = s >= start;
                    const unsigned long long cls = occ < 0 ? (hi ? 0ull : 2ull) : (hi ? 1ull : 3ull);
                    const unsigned long long l = occ < 0 ? 0ull : (unsigned long long)lu[s];
                    k = (cls << 62) | (l << 24) | (unsigned long long)s;
                }
                keys[s] = k;
            }
            __syncthreads();
            for (int size = 2; size <= S2; size <<= 1)
                for (int stride = size >> 1; stride > 0; stride >>= 1) {
                    for (int i = tid; i < (S2 >> 1); i += nthr) {
                        const int lo = 2 * i - (i & (stride - 1)), hi = lo + stride;
                        const bool up = ((lo & size) == 0);
                        const unsigned long long a = keys[lo], b = keys[hi];
                        if ((a > b) == up) keys[lo] = b, keys[hi] = a;
                    }
                    __syncthreads();
                }
            for (int j = tid; j < nmiss; j += nthr) {
                const int r = miss_r[j], e = uniq[r];
                const int s = (int)(keys[j] & 0xffffffull);
                const int ev = ris[s];
                uslot[r] = s;
                if (ev >= 0) F.rp.t.slot_of_real[ev] = -1;
                F.rp.t.real_in_slot[s] = id_base + e;
                lu[j] = (uint32_t)ev;  // the evicted id, for the miss list after the wait
            }
            __syncthreads();
        }
        // write back: this layer's tables, slot ids and weights (the miss list, shared by the
        // layers and read by the FFN before this kernel, is written after the wait)
        for (int r = tid; r < nuniq; r += nthr) {
            const int e = uniq[r], s = uslot[r];
            F.rp.t.slot_of_real[id_base + e] = s;
            F.rp.t.slot_last_used[s] = step;
        }
        for (int p = tid; p < n; p += nthr) {
            const int sl = sids[p] >= 0 ? uslot[first[sids[p]]] : -1;
            sids[p] = sl;
            F.rp.out[p] = sl;
            F.weights[p] = sw[p];
        }
        if (tid == 0) *F.rp.t.current_step = step;
    }
    auto write_counts = [&]() {
        if (tid == 0) {
            F.rp.m.counts[0] = status == NVMOE_ERR_BAD_EXPERT_ID ? 0 : nuniq;
            F.rp.m.counts[1] = status == NVMOE_OK ? nmiss : 0;
            F.rp.m.counts[2] = status;
            F.rp.m.counts[3] = n;
        }
    };
    int* hdr = wsp<int>(P, P.L.hdr);
    if (status != NVMOE_OK) {  // the FFN gets nothing to do (y = 0) and the status
        grid_dep_wait();  // (the error path waits in either mode)
        write_counts();
        if (tid == 0) {
            hdr[HDR_N_GROUPS] = 0;
            hdr[HDR_N_ACTIVE] = 0;
            hdr[HDR_N_ENT] = 0;
            hdr[HDR_STATUS] = status;
            if (P.status) *P.status = status;
        }
        return;
    }
    __syncthreads();

    // ---- C. FFN grouping from the slot ids, in shared memory (ffn_group_block, staged).
    // Groups in the order: hit slots, the shared expert, slots refilled in this step (so the
    // FFN's refill copies overlap the rest).
    int* missof = ris;  // miss index of each slot, -1: hit (the real_in_slot copy is done with)
    for (int s = tid; s < S; s += nthr) missof[s] = -1;
    __syncthreads();
    for (int j = tid; j < nmiss; j += nthr) missof[uslot[miss_r[j]]] = j;
    for (int p = tid; p < n; p += nthr)
        if (sids[p] >= 0) atomicAdd(&cnt[sids[p]], 1);
    __syncthreads();
    const int ngs = P.has_shared ? (n_tok + P.grp_tok - 1) / P.grp_tok : 0;
    // Entry, group and active-slot offsets of every slot (hit slots first, then the shared
    // expert's groups, then the slots refilled in this step), with two packed scans:
    // f: entries / groups of hit slots in bits 0-15 / 16-31, of missed slots in 32-47 / 48-63;
    // a: active hit / missed slots in bits 0-31 / 32-63 (every total is at most n <= 8192).
    // Slots past the first nthr keep their within-class rank in act / gbase / aidx until the
    // class totals are known.
    unsigned long long run_f = 0, run_a = 0;
    for (int base = 0; base < S; base += nthr) {
        const int s = base + tid;
        const int c = s < S ? cnt[s] : 0;
        const bool miss = s < S && missof[s] >= 0;
        const unsigned long long ng = (unsigned long long)((c + P.grp_tok - 1) / P.grp_tok);
        const int sh = miss ? 32 : 0;
        const unsigned long long f = ((unsigned long long)c | (ng << 16)) << sh;
        const unsigned long long av = (c > 0 ? 1ull : 0ull) << sh;
        unsigned long long tf, ta;
        const unsigned long long xf = block_exclusive_scan_u64(f, warp_sums64, &tf) + run_f;
        const unsigned long long xa = block_exclusive_scan_u64(av, warp_sums64, &ta) + run_a;
        run_f += tf;
        run_a += ta;
        if (s < S) {
            act[s] = c > 0 ? (int)((xf >> sh) & 0xffff) : -1;  // entry rank within the class
            gbase[s] = (int)((xf >> (sh + 16)) & 0xffff);
            aidx[s] = (int)((xa >> sh) & 0xffffffffu);
            cnt[s] = c;
        }
    }
    const int ent_hit = (int)(run_f & 0xffff), grp_hit = (int)((run_f >> 16) & 0xffff);
    const int act_hit = (int)(run_a & 0xffffffffu);
    const int g_shared = grp_hit;
    int n_act = act_hit + (int)(run_a >> 32);
    int n_ent = ent_hit + (int)((run_f >> 32) & 0xffff);
    const int n_grp = grp_hit + ngs + (int)(run_f >> 48);
    for (int s = tid; s < S; s += nthr) {
        const bool miss = missof[s] >= 0;
        if (act[s] >= 0) {
            act[s] += miss ? ent_hit : 0;     // entry base of the slot
            cnt[s] = act[s];                  // scatter cursor
        }
        gbase[s] += miss ? grp_hit + ngs : 0;  // first group of the slot
        aidx[s] += miss ? act_hit : 0;         // its place in the active-slot list
    }
    __syncthreads();
    for (int p = tid; p < n; p += nthr) {
        if (sids[p] < 0) {
            pe[p] = -1;
            continue;
        }
        const int e = atomicAdd(&cnt[sids[p]], 1);
        ent_tok_s[e] = p / K;
        ent_w_s[e] = sw[p];
        pe[p] = e;
    }
    __syncthreads();

    // ---- D. the miss list, token rows and the FFN workspace: after the previous kernel, or
    // (early outputs: a set of buffers the kernel in flight does not use) right away, with the
    // wait at the end, so that this kernel still completes only after the one before it
    if (!F.early) grid_dep_wait();
    {
        const nvmoe_miss_list& M = F.rp.m;
        for (int r = tid; r < nuniq; r += nthr) {
            M.unique_ids[r] = uniq[r];
            M.unique_slot[r] = uslot[r];
            M.unique_hit[r] = missof[uslot[r]] < 0 ? 1 : 0;
        }
        for (int j = tid; j < nmiss; j += nthr) {
            const int r = miss_r[j];
            M.miss_ids[j] = uniq[r];
            M.miss_slots[j] = uslot[r];
            M.evicted_ids[j] = (int)lu[j];
        }
        write_counts();
    }
    reset_phase_counters(P);
    for (int t = warp; t < n_tok; t += nw) {
        // a pre-routed token with no entry (and no shared expert) is not read by the FFN
        bool used = F.logits != nullptr || P.has_shared;
        for (int j = lane; j < K && !used; j += 32) used = sids[t * K + j] >= 0;
        if (!__any_sync(0xffffffffu, used)) continue;
        front_convert_token(P, t, lane);
    }
    int* desc = wsp<int>(P, P.L.grp_desc);
    int* ent_of = wsp<int>(P, P.L.ent_of);
    for (int s = tid; s < S; s += nthr) {  // the routed groups' records
        const int eb = act[s];
        if (eb < 0) continue;
        const int c = cnt[s] - eb;  // the cursor ended at base + count
        wsp<int>(P, P.L.active_slot)[aidx[s]] = s;
        wsp<int>(P, P.L.tok_cnt)[aidx[s]] = c;
        for (int i = 0; i * P.grp_tok < c; ++i) {
            int* d = desc + (int64_t)(gbase[s] + i) * kDescInts;
            d[GD_SLOT] = s;
            d[GD_POOL] = 0;
            d[GD_E0] = eb + i * P.grp_tok;
            d[GD_NT] = min(P.grp_tok, c - i * P.grp_tok);
            finish_record(P, gbase[s] + i, d, ent_tok_s + eb + i * P.grp_tok,
                          ent_w_s + eb + i * P.grp_tok);
            if (P.rf.n_banks > 0) d[GD_MISS] = missof[s] + 1;
        }
    }
    for (int j = tid; j < 2 * nmiss; j += nthr) wsp<int>(P, P.L.rdy)[j] = 0;
    for (int p = tid; p < n; p += nthr) {
        const int t = p / K, j = p - t * K;
        ent_of[t * (K + 1) + j] = pe[p];
    }
    for (int e = tid; e < n_ent; e += nthr) {
        wsp<int>(P, P.L.ent_tok)[e] = ent_tok_s[e];
        wsp<float>(P, P.L.ent_w)[e] = ent_w_s[e];
    }
    if (P.has_shared) {
        for (int t = tid; t < n_tok; t += nthr) {
            const int e = n_ent + t;
            wsp<int>(P, P.L.ent_tok)[e] = t;
            wsp<float>(P, P.L.ent_w)[e] = 1.0f;
            ent_of[t * (K + 1) + K] = e;
        }
        for (int i = tid; i < ngs; i += nthr) {
            int* d = desc + (int64_t)(g_shared + i) * kDescInts;
            const int nt = min(P.grp_tok, n_tok - i * P.grp_tok);
            d[GD_SLOT] = 0;
            d[GD_POOL] = 1;
            d[GD_E0] = n_ent + i * P.grp_tok;
            d[GD_NT] = nt;
            int toks[kGroupMaxTok];
#pragma unroll
            for (int k = 0; k < kGroupMaxTok; ++k) toks[k] = i * P.grp_tok + k;
            finish_record(P, g_shared + i, d, toks, nullptr);
        }
        if (tid == 0) {
            wsp<int>(P, P.L.active_slot)[n_act] = 0;
            wsp<int>(P, P.L.tok_cnt)[n_act] = n_tok;
        }
        n_act += 1;
        n_ent += n_tok;
    } else {
        for (int t = tid; t < n_tok; t += nthr) ent_of[t * (K + 1) + K] = -1;
    }
    if (tid == 0) {
        hdr[HDR_N_GROUPS] = n_grp;
        hdr[HDR_N_ACTIVE] = n_act;
        hdr[HDR_N_ENT] = n_ent;
        hdr[HDR_STATUS] = NVMOE_OK;
        if (P.status) *P.status = NVMOE_OK;
    }
    if (F.early) grid_dep_wait();
}

}  // namespace

int ffn_launch_main(FfnParams& P, cudaStream_t st);
int ffn_setup(const nvmoe_ffn_args* args, FfnParams& P);

}  // namespace nvmoe

extern "C" int nvmoe_decode_layer(const nvmoe_decode_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->slot_ids || !a->weights) return NVMOE_ERR_INVALID_ARG;
    const nvmoe_slot_table& t = a->table;
    if (!t.slot_of_real || !t.real_in_slot || !t.slot_last_used || !t.current_step)
        return NVMOE_ERR_INVALID_ARG;
    if (t.n_expert <= 0 || t.n_expert > kMaxExperts || t.cache_size <= 0 ||
        t.cache_size > kMaxSlotsRemap || t.pinned_k < 0 || t.id_base < 0)
        return NVMOE_ERR_INVALID_ARG;
    if (a->top_k <= 0 || a->top_k > kMaxTopK || a->top_k > t.n_expert || a->n_tok < 0)
        return NVMOE_ERR_INVALID_ARG;
    if (a->router_mode != NVMOE_ROUTER_SOFTMAX && a->router_mode != NVMOE_ROUTER_SIGMOID_BIAS)
        return NVMOE_ERR_INVALID_ARG;
    if (!a->logits && (!a->routed_ids || !a->routed_weights)) return NVMOE_ERR_INVALID_ARG;
    const nvmoe_miss_list& m = a->misses;
    if (!m.unique_ids || !m.unique_slot || !m.unique_hit || !m.miss_ids || !m.miss_slots ||
        !m.evicted_ids || !m.counts)
        return NVMOE_ERR_INVALID_ARG;
    const int64_t n = (int64_t)a->n_tok * a->top_k;
    if (m.capacity < std::min<int64_t>(n, t.n_expert)) return NVMOE_ERR_INVALID_ARG;
    if (a->ffn.pool && a->ffn.pool->n_slots < t.cache_size) return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok == 0) return NVMOE_OK;

    nvmoe_ffn_args fa = a->ffn;
    fa.slot_ids = a->slot_ids;
    fa.ids_row_stride = a->top_k;
    fa.weights = a->weights;
    fa.weights_row_stride = a->top_k;
    fa.top_k = a->top_k;
    fa.n_tok = a->n_tok;
    FrontParams F;
    int rc = ffn_setup(&fa, F.fp);
    if (rc != NVMOE_OK) return rc;
    F.logits = a->logits;
    F.lstride = a->logits_row_stride;
    F.mode = a->router_mode;
    F.bias = a->router_bias;
    F.norm_topk = a->norm_topk;
    F.scaling = a->routed_scaling;
    F.weights = a->weights;
    F.rp.t = t;
    F.rp.ids = a->slot_ids;
    F.rp.ids_stride = (int64_t)a->top_k * 4;
    F.rp.out = a->slot_ids;
    F.rp.out_stride = (int64_t)a->top_k * 4;
    F.rp.top_k = a->top_k;
    F.rp.n_tok = a->n_tok;
    F.rp.is_decode = a->is_decode;
    F.rp.m = m;
    F.early = a->early_outputs ? 1 : 0;
    F.inputs_after_wait = a->inputs_after_wait ? 1 : 0;
    F.rids = a->routed_ids;
    F.rw = a->routed_weights;
    F.rstride = a->routed_row_stride > 0 ? a->routed_row_stride : a->top_k;

    if (n > kFrontMaxIds || t.cache_size > kFrontMaxSlots) return NVMOE_ERR_UNSUPPORTED;
    if (F.fp.pool.n_slots < t.cache_size) return NVMOE_ERR_INVALID_ARG;
    const size_t smem = (size_t)front_smem(t.n_expert, t.cache_size, (int)n, (int)n + a->n_tok).total;
    if (smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream;
    F.fp.spare_sm = 1;
    // The mma.sync FFN copies the misses in itself, overlapped with the hit groups; the FP4
    // tensor-core FFN runs after a separate gather kernel.
    bool in_kernel_refill = false;
    if (a->refill_banks && a->n_refill_banks > 0) {
        if (!a->host_slot_of_id || !m.miss_ids || !m.miss_slots) return NVMOE_ERR_INVALID_ARG;
        for (int b = 0; b < a->n_refill_banks; ++b) {
            const nvmoe_refill_bank& B = a->refill_banks[b];
            if (!B.dst || !B.src || B.row_bytes < 0) return NVMOE_ERR_INVALID_ARG;
        }
        if (!F.fp.use_fp4 && a->n_refill_banks <= kRefillMaxBanks) {
            FfnRefill& R = F.fp.rf;
            R.n_banks = a->n_refill_banks;
            R.pbase[0] = 0;
            // the gate/up banks first: a missed group's gate_up starts once they are in
            const nvmoe_matrix_bank& dn = F.fp.pool.down;
            auto is_down = [&](const nvmoe_refill_bank& B) {
                return B.dst == dn.data || (dn.scale && B.dst == dn.scale) ||
                       (dn.global_scale && B.dst == (const void*)dn.global_scale);
            };
            int order[kRefillMaxBanks], no = 0;
            for (int ph = 0; ph < 2; ++ph)
                for (int b = 0; b < R.n_banks; ++b)
                    if ((int)is_down(a->refill_banks[b]) == ph) order[no++] = b;
            R.pieces_gu = R.pieces_dn = 0;
            for (int b = 0; b < R.n_banks; ++b) {
                const nvmoe_refill_bank& B = a->refill_banks[order[b]];
                R.banks[b] = B;
                R.down[b] = is_down(B) ? 1 : 0;
                const uint64_t bits = (uint64_t)B.row_bytes | (uint64_t)B.dst_slot_stride |
                                      (uint64_t)B.src_slot_stride |
                                      reinterpret_cast<uintptr_t>(B.dst) |
                                      reinterpret_cast<uintptr_t>(B.src);
                R.vec16[b] = (bits & 15) == 0;  // pieces start at multiples of 16 bytes
                R.vec4[b] = (bits & 3) == 0;
                const int pcs = (int)((B.row_bytes + kRefillPiece - 1) / kRefillPiece);
                R.pbase[b + 1] = R.pbase[b] + pcs;
                (R.down[b] ? R.pieces_dn : R.pieces_gu) += pcs;
            }
            R.counts = m.counts;
            R.miss_ids = m.miss_ids;
            R.miss_slots = m.miss_slots;
            R.host_slot_of_id = a->host_slot_of_id;
            R.n_gpu_slots = t.cache_size;
            in_kernel_refill = true;
        }
    }
    if (smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(decode_front_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    // 8 warps up to 8 tokens, 16 above: routing warps plus token-conversion warps
    const int threads = a->n_tok <= 8 ? 256 : kFrontThreads;
    cudaError_t e = launch_pdl(decode_front_kernel, dim3(1), dim3(threads), smem, st, true, F);
    if (e != cudaSuccess) return cuda_status("decode_front launch", e);
    if (a->refill_banks && a->n_refill_banks > 0 && !in_kernel_refill) {
        rc = nvmoe_refill_gather(a->refill_banks, a->n_refill_banks, &a->misses,
                                 a->host_slot_of_id, t.cache_size, stream);
        if (rc != NVMOE_OK) return rc;
    }
    return ffn_launch_main(F.fp, st);
}
