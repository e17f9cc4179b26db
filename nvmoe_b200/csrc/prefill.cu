// R10 — prefill: the routed-expert FFN for large batches as a token-sorted grouped GEMM on the
// 5th-generation tensor cores (tcgen05, accumulators in tensor memory).
//
// Reference: the narrowed-union prefill patch (nvme-moe-bench/nvme_offload_cache.py:1957-2013:
// union of the routed ids -> ensure -> _expert_gemm over the slot pool with is_prefill) and
// llama.cpp's mul_mat_id over the reduced expert tensors for n_tokens > 1 (eval_cb with the
// ubatch clamp, scripts/moe_cache_probe.cpp:1668-1684).  Same result as the decode kernel:
//   y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] ),  s = slot_ids[t, j]
// plus the shared expert (weight 1, or sigmoid(x . shared_gate)).
//
// Steps (one stream, all device-side):
//   count   — entries per slot (the shared expert is one more key holding every token)
//   scan    — entry base per key, tiles of <= 128 entries per key
//   scatter — entries sorted by key; inverse map ent_of[t * (k + 1) + j]
//   gather  — the sorted activation matrix xs[e] = f16(x[tok(e)]) and the shared gate
//   gate_up — one CTA per (tile half, 128 rows of I): D_g = W_g xs^T and D_u = W_u xs^T with the
//             weights dequantised by the CTA's warps straight into tensor memory (A operand),
//             xs from shared memory (B operand), fp32 accumulators in tensor memory;
//             h = silu(g * global_g) * (u * global_u) (f16)
//   down    — one CTA per (tile, 128 rows of H): y_part[e] = w_e * down(h_e) (fp32)
//   combine — y[t] = sum over t's entries in the order j = 0..k-1, shared (bf16)
// Deterministic: no floating-point atomics.
#include "common.cuh"
#include "umma.cuh"
#include "ffn_common.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace nvmoe {
namespace {

constexpr int kTileN = 128;   // entries per tile (the MMA N)
constexpr int kTileM = 128;   // weight rows per CTA (the MMA M)
constexpr int kChunk = 64;    // K values per pipeline stage
constexpr int kPfThreads = 256;

enum { PH_N_TILES = 0, PH_N_ENT = 1, PH_STATUS = 2 };

struct PfLayout {
    size_t hdr, cnt, base, cursor, tile_base, tiles, ent_tok, ent_w, ent_of, sg, xs, h, ypart,
        total;
    int n_keys, n_ent_max, max_tiles;
};

__host__ __device__ inline PfLayout pf_layout(int n_tok, int top_k, int H, int I, int n_slots) {
    PfLayout L;
    L.n_keys = n_slots + 1;  // the shared expert is key n_slots
    L.n_ent_max = n_tok * (top_k + 1);
    L.max_tiles = (L.n_ent_max + kTileN - 1) / kTileN + std::min(L.n_keys, L.n_ent_max);
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 256);
        return at;
    };
    L.hdr = take(64);
    L.cnt = take(4 * (size_t)L.n_keys);
    L.base = take(4 * (size_t)L.n_keys);
    L.cursor = take(4 * (size_t)L.n_keys);
    L.tile_base = take(4 * (size_t)L.n_keys);
    L.tiles = take(12 * (size_t)L.max_tiles);  // {key, entry base, rows}
    L.ent_tok = take(4 * (size_t)L.n_ent_max);
    L.ent_w = take(4 * (size_t)L.n_ent_max);
    L.ent_of = take(4 * (size_t)L.n_ent_max);
    L.sg = take(4 * (size_t)n_tok);
    L.xs = take(2 * (size_t)L.n_ent_max * H);
    L.h = take(2 * (size_t)L.n_ent_max * I);
    L.ypart = take(4 * (size_t)L.n_ent_max * H);
    L.total = o;
    return L;
}

struct PfParams {
    nvmoe_expert_pool pool, shared;
    int has_shared;
    const uint16_t* shared_gate;
    const uint16_t* x;
    int64_t x_stride;
    const int32_t* ids;
    int64_t ids_stride;
    const float* w;
    int64_t w_stride;
    int top_k, n_tok;
    uint16_t* y;
    int64_t y_stride;
    unsigned char* ws;
    PfLayout L;
    int32_t* status;
};

template <typename T>
__device__ __forceinline__ T* pws(const PfParams& P, size_t off) {
    return reinterpret_cast<T*>(P.ws + off);
}

// ------------------------------------------------------------------ grouping
__global__ void pf_count(PfParams P) {
    const int n = P.n_tok * P.top_k, S = P.pool.n_slots;
    int* cnt = pws<int>(P, P.L.cnt);
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const int t = p / P.top_k, j = p - t * P.top_k;
        const int s = P.ids[(int64_t)t * P.ids_stride + j];
        if (s >= 0 && s < S)
            atomicAdd(&cnt[s], 1);
        else if (s >= S)  // (a negative id is an empty entry)
            atomicExch(pws<int>(P, P.L.hdr) + PH_STATUS, NVMOE_ERR_BAD_SLOT);
    }
}

// One block: entry bases (exclusive scan over keys) and the tile list.
__global__ void __launch_bounds__(1024) pf_scan(PfParams P) {
    __shared__ int warp_sums[33];
    const int K = P.L.n_keys, S = P.pool.n_slots, tid = threadIdx.x;
    int* cnt = pws<int>(P, P.L.cnt);
    int* base = pws<int>(P, P.L.base);
    int* cursor = pws<int>(P, P.L.cursor);
    int* tile_base = pws<int>(P, P.L.tile_base);
    int* tiles = pws<int>(P, P.L.tiles);
    if (tid == 0) cnt[S] = P.has_shared ? P.n_tok : 0;
    __syncthreads();
    int run_e = 0, run_t = 0;
    for (int b0 = 0; b0 < K; b0 += blockDim.x) {
        const int s = b0 + tid;
        const int c = s < K ? cnt[s] : 0;
        const int nt = (c + kTileN - 1) / kTileN;
        int tot_e, tot_t;
        const int re = block_exclusive_scan(c, warp_sums, &tot_e);
        const int rt = block_exclusive_scan(nt, warp_sums, &tot_t);
        if (s < K) {
            base[s] = run_e + re;
            cursor[s] = run_e + re;
            tile_base[s] = run_t + rt;
            for (int i = 0; i < nt; ++i) {
                int* tl = tiles + 3 * (run_t + rt + i);
                tl[0] = s;
                tl[1] = run_e + re + i * kTileN;
                tl[2] = min(kTileN, c - i * kTileN);
            }
        }
        run_e += tot_e;
        run_t += tot_t;
    }
    if (tid == 0) {
        int* hdr = pws<int>(P, P.L.hdr);
        hdr[PH_N_TILES] = run_t;
        hdr[PH_N_ENT] = run_e;
    }
}

__global__ void pf_scatter(PfParams P) {
    const int S = P.pool.n_slots, K1 = P.top_k + 1;
    int* cursor = pws<int>(P, P.L.cursor);
    const int* base = pws<int>(P, P.L.base);
    int* ent_tok = pws<int>(P, P.L.ent_tok);
    float* ent_w = pws<float>(P, P.L.ent_w);
    int* ent_of = pws<int>(P, P.L.ent_of);
    const int n = P.n_tok * K1;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const int t = p / K1, j = p - t * K1;
        int e = -1;
        if (j < P.top_k) {
            const int s = P.ids[(int64_t)t * P.ids_stride + j];
            if (s >= 0 && s < S) {
                e = atomicAdd(&cursor[s], 1);  // order inside a key does not change any result
                ent_tok[e] = t;
                ent_w[e] = P.w[(int64_t)t * P.w_stride + j];
            }
        } else if (P.has_shared) {
            e = base[S] + t;
            ent_tok[e] = t;
            ent_w[e] = 1.0f;
        }
        ent_of[p] = e;
    }
}

// One block per entry: xs[e] = f16(x[tok]); for the shared key also sg[tok] = sigmoid(x . g).
__global__ void __launch_bounds__(128) pf_gather(PfParams P) {
    const int H = P.pool.hidden, S = P.pool.n_slots;
    const int n_ent = pws<int>(P, P.L.hdr)[PH_N_ENT];
    const int e = blockIdx.x;
    if (e >= n_ent) return;
    const int t = pws<int>(P, P.L.ent_tok)[e];
    const uint16_t* xr = P.x + (int64_t)t * P.x_stride;
    __half* xs = pws<__half>(P, P.L.xs) + (int64_t)e * H;
    const bool gate = P.has_shared && P.shared_gate && e >= pws<int>(P, P.L.base)[S];
    float dot = 0.f;
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
        const uint16_t* u = reinterpret_cast<const uint16_t*>(&v);
        __align__(16) __half o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float f = bf16_bits_to_f32(u[k]);
            o[k] = __float2half_rn(f);
            if (gate) dot = fmaf(f, bf16_bits_to_f32(P.shared_gate[i + k]), dot);
        }
        *reinterpret_cast<uint4*>(xs + i) = *reinterpret_cast<const uint4*>(o);
    }
    if (gate) {
        __shared__ float red[4];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
        if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dot;
        __syncthreads();
        if (threadIdx.x == 0)
            pws<float>(P, P.L.sg)[t] = 1.0f / (1.0f + expf(-(red[0] + red[1] + red[2] + red[3])));
    }
}

// ------------------------------------------------------------------ tensor-core GEMM pieces
// 64 NVFP4 values of one row (32 code bytes, 4 E4M3 scales) -> 32 f16x2 words, K ascending.
__device__ __forceinline__ void deq_row64(const uint4 (&c)[2], uint32_t sc4, uint32_t (&o)[32]) {
    const uint32_t s01 = e4m3x2_to_f16x2((uint16_t)(sc4 & 0xffff));
    const uint32_t s23 = e4m3x2_to_f16x2((uint16_t)(sc4 >> 16));
    const uint32_t sc[4] = {prmt(s01, 0, 0x1010), prmt(s01, 0, 0x3232), prmt(s23, 0, 0x1010),
                            prmt(s23, 0, 0x3232)};
    const uint32_t w[8] = {c[0].x, c[0].y, c[0].z, c[0].w, c[1].x, c[1].y, c[1].z, c[1].w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {  // word i = K 8i .. 8i+7, scale block i / 2
        uint32_t a0, a1, a2, a3;
        asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
            "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
            "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
            "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
            "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
            "cvt.rn.f16x2.e2m1x2 %3, b3; }"
            : "=r"(a0), "=r"(a1), "=r"(a2), "=r"(a3)
            : "r"(w[i]));
        const uint32_t s = sc[i >> 1];
        o[4 * i + 0] = hmul2_u32(a0, s);
        o[4 * i + 1] = hmul2_u32(a1, s);
        o[4 * i + 2] = hmul2_u32(a2, s);
        o[4 * i + 3] = hmul2_u32(a3, s);
    }
}

struct RowSrc {
    const uint8_t* codes;   // row start
    const uint8_t* scales;  // row start
};

__device__ __forceinline__ RowSrc row_src(const nvmoe_matrix_bank& b, int slot, int64_t row) {
    RowSrc r;
    r.codes = (const uint8_t*)b.data + slot * b.slot_stride + row * b.row_stride;
    r.scales = (const uint8_t*)b.scale + slot * b.scale_slot_stride + row * b.scale_row_stride;
    return r;
}

// Ampere-style asynchronous copies (per thread, into shared memory).
__device__ __forceinline__ void cp16(void* dst, const void* src, int src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
                 "r"(src_bytes)
                 : "memory");
}
__device__ __forceinline__ void cp4(void* dst, const void* src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(dst)), "l"(src)
                 : "memory");
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Pipeline: kStages shared-memory stages, loads issued kStages - 2 chunks ahead; a stage and the
// TMEM A buffer of chunk c are reused by chunk c + 2 once chunk c's MMAs have completed.
// Four stages keep two CTAs per SM, so one CTA's prologue and epilogue overlap the other's MMAs.
constexpr int kStages = 4;

// B chunk c: rows [eb, eb + nr) of a row-major f16 matrix (row length ld) into the canonical
// layout of an NB-row tile; rows >= nr are zero.
template <int NB>
__device__ __forceinline__ void issue_b(uint8_t* dst, const __half* m, int64_t ld, int eb, int nr,
                                        int c) {
#pragma unroll
    for (int u = 0; u < NB * 8 / kPfThreads; ++u) {
        const int p = threadIdx.x + kPfThreads * u;
        const int n = p >> 3, kp = p & 7;
        const bool v = n < nr;
        cp16(dst + umma::canon_off(n, kp * 8, NB),
             m + (int64_t)(eb + (v ? n : 0)) * ld + c * kChunk + kp * 8, v ? 16 : 0);
    }
}

// The tail of a chunk: make this thread's TMEM stores and async copies visible to the MMA, then
// one thread issues the chunk's K-steps (A columns a_col[j] + 8 ks for each accumulator j).
template <int NB, int NACC>
__device__ __forceinline__ void chunk_mma(uint8_t* bstage, const uint32_t (&d)[NACC],
                                          const uint32_t (&a_col)[NACC], int c, uint64_t* done) {
    umma::wait_st();
    umma::fence_smem_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (threadIdx.x == 0) {
        constexpr uint32_t idesc = umma::idesc_f16(kTileM, NB);
        const uint32_t b0 = smem_u32(bstage);
#pragma unroll
        for (int ks = 0; ks < kChunk / 16; ++ks) {
            const uint64_t bd = umma::smem_desc(b0 + ks * 2 * (NB / 8) * 128, (NB / 8) * 128, 128);
#pragma unroll
            for (int j = 0; j < NACC; ++j)
                umma::mma_ts(d[j], a_col[j] + 8 * ks, bd, idesc, (c > 0 || ks > 0) ? 1u : 0u);
        }
        umma::commit(done);
    }
}

// gate_up.  One CTA per (tile, 128 rows of I, half of the tile's entries): N = 64 keeps the
// CTA's tensor memory at 256 columns (two CTAs per SM).  Per stage: codes [256 rows][32 B]
// (rows 0-127 gate, 128-255 up; row = thread), scales [256][4 B], B [64 x 64 f16].  TMEM: D_g
// [0,64), D_u [64,128), A buffer b: gate [128 + 64 b, +32), up [160 + 64 b, +32).  Warps 0-3
// dequantise gate rows, warps 4-7 up rows.
constexpr int kGuN = 64;
constexpr int kGuCodes = 2 * kTileM * 32, kGuScales = 2 * kTileM * 4;
constexpr int kGuStage = kGuCodes + kGuScales + kGuN * kChunk * 2;

__global__ void __launch_bounds__(kPfThreads, 1) pf_gate_up(PfParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t mma_done[2];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int* hdr = pws<int>(P, P.L.hdr);
    const int tile = blockIdx.x, mt = blockIdx.y;
    if (tile >= hdr[PH_N_TILES]) return;
    const int* tl = pws<int>(P, P.L.tiles) + 3 * tile;
    const int key = tl[0];
    const int eb = tl[1] + kGuN * blockIdx.z, nr = min(kGuN, tl[2] - kGuN * (int)blockIdx.z);
    if (nr <= 0) return;
    const int H = P.pool.hidden, I = P.pool.inter, S = P.pool.n_slots;
    const bool sh = key == S;
    const nvmoe_expert_pool& pool = sh ? P.shared : P.pool;
    const int slot = sh ? 0 : key;
    const int row = (warp & 3) * 32 + lane;
    const bool is_up = warp >= 4;
    const RowSrc src = row_src(is_up ? pool.up : pool.gate, slot, (int64_t)mt * kTileM + row);
    const __half* xs = pws<__half>(P, P.L.xs);
    auto stage = [&](int c) { return smem + (size_t)(c % kStages) * kGuStage; };
    auto issue = [&](int c) {
        uint8_t* st = stage(c);
        cp16(st + tid * 32, src.codes + c * 32, 16);
        cp16(st + tid * 32 + 16, src.codes + c * 32 + 16, 16);
        cp4(st + kGuCodes + tid * 4, src.scales + c * 4);
        issue_b<kGuN>(st + kGuCodes + kGuScales, xs, H, eb, nr, c);
    };

    if (tid == 0) {
        mbar_init(&mma_done[0], 1);
        mbar_init(&mma_done[1], 1);
        mbar_init_fence();
    }
    if (warp == 0) umma::tmem_alloc(&tmem_base, 256);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tm = tmem_base;
    const uint32_t dd[2] = {tm, tm + kGuN};

    const int n_chunks = H / kChunk;
    for (int c = 0; c < kStages - 2; ++c) {
        if (c < n_chunks) issue(c);
        cp_commit();
    }
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
        if (c >= 2 && ok && !mbar_wait_bounded(&mma_done[c & 1], ((c - 2) >> 1) & 1)) ok = false;
        if (c + kStages - 2 < n_chunks) issue(c + kStages - 2);
        cp_commit();
        cp_wait<kStages - 2>();
        umma::fence_after_sync();
        const uint8_t* st = stage(c);
        uint4 cw[2];
        cw[0] = *reinterpret_cast<const uint4*>(st + tid * 32);
        cw[1] = *reinterpret_cast<const uint4*>(st + tid * 32 + 16);
        const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(st + kGuCodes + tid * 4);
        uint32_t a[32];
        deq_row64(cw, sc4, a);
        const uint32_t acol = 128 + 64 * (c & 1) + (is_up ? 32 : 0);
        uint32_t lo[16], hi[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lo[i] = a[i], hi[i] = a[16 + i];
        umma::st_x16(umma::lane_addr(tm, warp, acol), lo);
        umma::st_x16(umma::lane_addr(tm, warp, acol + 16), hi);
        const uint32_t ac[2] = {tm + 128 + 64 * (c & 1), tm + 160 + 64 * (c & 1)};
        chunk_mma<kGuN, 2>(const_cast<uint8_t*>(st) + kGuCodes + kGuScales, dd, ac, c,
                           &mma_done[c & 1]);
    }
    // the last commit covers every MMA of the tile
    const int last = n_chunks - 1;
    if (ok && !mbar_wait_bounded(&mma_done[last & 1], (last >> 1) & 1)) ok = false;
    umma::fence_after_sync();
    if (!ok) {
        if (lane == 0) atomicExch(pws<int>(P, P.L.hdr) + PH_STATUS, NVMOE_ERR_TIMEOUT);
    } else {
        // epilogue: warps 0-3 entries [0, 32), warps 4-7 entries [32, 64) of the rows they own
        const float gg = global_of(pool.gate, slot), ug = global_of(pool.up, slot);
        __half* h = pws<__half>(P, P.L.h);
        const int c0 = is_up ? kGuN / 2 : 0;
#pragma unroll 1
        for (int cc = c0; cc < c0 + kGuN / 2 && cc < nr; cc += 16) {
            uint32_t g[16], u[16];
            umma::ld_x16(umma::lane_addr(dd[0], warp, cc), g);
            umma::ld_x16(umma::lane_addr(dd[1], warp, cc), u);
            umma::wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int n = cc + i;
                if (n < nr)
                    h[(int64_t)(eb + n) * I + mt * kTileM + row] = __float2half_rn(
                        silu(__uint_as_float(g[i]) * gg) * (__uint_as_float(u[i]) * ug));
            }
        }
    }
    cp_wait<0>();
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tm, 256);
}

// down.  Per stage: codes [128 rows][32 B] (each thread copies its row's half: warps 0-3 K 0-31,
// warps 4-7 K 32-63), scales [128][4 B], B [128 x 64 f16] = h.  TMEM: D [0,128), A buffer b
// [128 + 32 b, +32).
constexpr int kDnCodes = kTileM * 32, kDnScales = kTileM * 4;
constexpr int kDnStage = kDnCodes + kDnScales + kTileN * kChunk * 2;

__global__ void __launch_bounds__(kPfThreads, 1) pf_down(PfParams P) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ __align__(8) uint64_t mma_done[2];
    __shared__ uint32_t tmem_base;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int* hdr = pws<int>(P, P.L.hdr);
    const int tile = blockIdx.x, mt = blockIdx.y;
    if (tile >= hdr[PH_N_TILES]) return;
    const int* tl = pws<int>(P, P.L.tiles) + 3 * tile;
    const int key = tl[0], eb = tl[1], nr = tl[2];
    const int H = P.pool.hidden, I = P.pool.inter, S = P.pool.n_slots;
    const bool sh = key == S;
    const nvmoe_expert_pool& pool = sh ? P.shared : P.pool;
    const int slot = sh ? 0 : key;
    const int row = (warp & 3) * 32 + lane;
    const int half = warp >= 4 ? 1 : 0;  // K half of each chunk
    const RowSrc src = row_src(pool.down, slot, (int64_t)mt * kTileM + row);
    const __half* hm = pws<__half>(P, P.L.h);
    auto stage = [&](int c) { return smem + (size_t)(c % kStages) * kDnStage; };
    auto issue = [&](int c) {
        uint8_t* st = stage(c);
        cp16(st + row * 32 + half * 16, src.codes + c * 32 + half * 16, 16);
        if (!half) cp4(st + kDnCodes + row * 4, src.scales + c * 4);
        issue_b<kTileN>(st + kDnCodes + kDnScales, hm, I, eb, nr, c);
    };

    if (tid == 0) {
        mbar_init(&mma_done[0], 1);
        mbar_init(&mma_done[1], 1);
        mbar_init_fence();
    }
    if (warp == 0) umma::tmem_alloc(&tmem_base, 256);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tm = tmem_base;
    const uint32_t dd[1] = {tm};

    const int n_chunks = I / kChunk;
    for (int c = 0; c < kStages - 2; ++c) {
        if (c < n_chunks) issue(c);
        cp_commit();
    }
    bool ok = true;
    for (int c = 0; c < n_chunks; ++c) {
        if (c >= 2 && ok && !mbar_wait_bounded(&mma_done[c & 1], ((c - 2) >> 1) & 1)) ok = false;
        if (c + kStages - 2 < n_chunks) issue(c + kStages - 2);
        cp_commit();
        cp_wait<kStages - 2>();
        __syncthreads();  // the scale bytes of a row are copied by the warp of its first half
        umma::fence_after_sync();
        const uint8_t* st = stage(c);
        uint4 cw[2];
        cw[0] = *reinterpret_cast<const uint4*>(st + row * 32 + half * 16);
        cw[1] = make_uint4(0, 0, 0, 0);
        const uint32_t sc4 = *reinterpret_cast<const uint32_t*>(st + kDnCodes + row * 4);
        uint32_t a[32];
        deq_row64(cw, half ? (sc4 >> 16) : (sc4 & 0xffff), a);  // first 16 words meaningful
        uint32_t lo[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) lo[i] = a[i];
        umma::st_x16(umma::lane_addr(tm, warp, 128 + 32 * (c & 1) + 16 * half), lo);
        const uint32_t ac[1] = {tm + 128 + 32 * (c & 1)};
        chunk_mma<kTileN, 1>(const_cast<uint8_t*>(st) + kDnCodes + kDnScales, dd, ac, c,
                             &mma_done[c & 1]);
    }
    const int last = n_chunks - 1;
    if (ok && !mbar_wait_bounded(&mma_done[last & 1], (last >> 1) & 1)) ok = false;
    umma::fence_after_sync();
    if (!ok) {
        if (lane == 0) atomicExch(pws<int>(P, P.L.hdr) + PH_STATUS, NVMOE_ERR_TIMEOUT);
    } else {
        const float dg = global_of(pool.down, slot);
        const float* ent_w = pws<float>(P, P.L.ent_w);
        const int* ent_tok = pws<int>(P, P.L.ent_tok);
        const float* sgv = (sh && P.shared_gate) ? pws<float>(P, P.L.sg) : nullptr;
        float* yp = pws<float>(P, P.L.ypart);
        const int c0 = half ? 64 : 0;
#pragma unroll 1
        for (int cc = c0; cc < c0 + 64 && cc < nr; cc += 16) {
            uint32_t d[16];
            umma::ld_x16(umma::lane_addr(tm, warp, cc), d);
            umma::wait_ld();
#pragma unroll
            for (int i = 0; i < 16; ++i) {
                const int n = cc + i;
                if (n < nr) {
                    const int e = eb + n;
                    float wgt = ent_w[e];
                    if (sgv) wgt *= sgv[ent_tok[e]];
                    yp[(int64_t)e * H + mt * kTileM + row] = __uint_as_float(d[i]) * dg * wgt;
                }
            }
        }
    }
    cp_wait<0>();
    umma::fence_before_sync();
    __syncthreads();
    if (warp == 0) umma::tmem_dealloc(tm, 256);
}

// y[t] = sum_j y_part[ent_of[t, j]] in the order j = 0..k-1, shared; 4 columns per thread.
__global__ void pf_combine(PfParams P) {
    const int H = P.pool.hidden, K1 = P.top_k + 1;
    const int* ent_of = pws<int>(P, P.L.ent_of);
    const float* yp = pws<float>(P, P.L.ypart);
    const int64_t n4 = (int64_t)P.n_tok * (H / 4);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (H / 4)), c = (int)(i % (H / 4)) * 4;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < K1; ++j) {
            const int e = ent_of[t * K1 + j];
            if (e < 0) continue;
            const float4 v = *reinterpret_cast<const float4*>(yp + (int64_t)e * H + c);
            s.x += v.x, s.y += v.y, s.z += v.z, s.w += v.w;
        }
        uint2 o;
        o.x = (uint32_t)f32_to_bf16_bits(s.x) | ((uint32_t)f32_to_bf16_bits(s.y) << 16);
        o.y = (uint32_t)f32_to_bf16_bits(s.z) | ((uint32_t)f32_to_bf16_bits(s.w) << 16);
        *reinterpret_cast<uint2*>(P.y + (int64_t)t * P.y_stride + c) = o;
    }
}

__global__ void pf_status(PfParams P) {
    if (P.status) *P.status = pws<int>(P, P.L.hdr)[PH_STATUS];
}

bool pf_pool_ok(const nvmoe_expert_pool& p, int H, int I) {
    auto bank_ok = [](const nvmoe_matrix_bank& b, int k) {
        // 16-byte code loads at every 64-value chunk, 4-byte scale loads
        return b.data && b.scale && (reinterpret_cast<uintptr_t>(b.data) & 15) == 0 &&
               (reinterpret_cast<uintptr_t>(b.scale) & 3) == 0 && b.slot_stride % 16 == 0 &&
               b.row_stride % 16 == 0 && b.scale_slot_stride % 4 == 0 &&
               b.scale_row_stride % 4 == 0 && b.row_stride >= k / 2 &&
               b.scale_row_stride >= k / 16;
    };
    return p.quant == NVMOE_Q_NVFP4 && p.hidden == H && p.inter == I && p.n_slots > 0 &&
           bank_ok(p.gate, H) && bank_ok(p.up, H) && bank_ok(p.down, I);
}

}  // namespace

bool prefill_fp4_ok(const nvmoe_ffn_args* a);
size_t prefill_fp4_workspace(int n_tok, int top_k, int H, int I, int n_slots);
int prefill_fp4_run(const nvmoe_ffn_args* a, cudaStream_t st);

// The block-scaled FP4 path (prefill_fp4.cu) runs when the shapes suit it, unless the call
// asks for this file's kind::f16 path (nvmoe_ffn_args.kernel == NVMOE_KERNEL_F16).
bool prefill_use_fp4(const nvmoe_ffn_args* a) {
    return a->kernel != NVMOE_KERNEL_F16 && prefill_fp4_ok(a);
}

}  // namespace nvmoe

extern "C" size_t nvmoe_moe_ffn_prefill_workspace_size(int n_tok, int top_k, int hidden, int inter,
                                                        int n_slots) {
    const size_t f16 = nvmoe::pf_layout(std::max(n_tok, 1), top_k, hidden, inter, n_slots).total;
    const size_t fp4 = (hidden % 512 == 0 && inter % 256 == 0)
                           ? nvmoe::prefill_fp4_workspace(n_tok, top_k, hidden, inter, n_slots)
                           : 0;
    return std::max(f16, fp4);
}

extern "C" int nvmoe_moe_ffn_prefill(const nvmoe_ffn_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->pool || !a->x || !a->slot_ids || !a->weights || !a->y)
        return NVMOE_ERR_INVALID_ARG;
    const nvmoe_expert_pool& pool = *a->pool;
    const int H = pool.hidden, I = pool.inter;
    if (pool.quant != NVMOE_Q_NVFP4) return NVMOE_ERR_UNSUPPORTED;
    if (H % kTileM != 0 || I % kTileM != 0 || H % kChunk != 0 || I % kChunk != 0)
        return NVMOE_ERR_UNSUPPORTED;
    if (!pf_pool_ok(pool, H, I) || (a->shared && !pf_pool_ok(*a->shared, H, I)))
        return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok < 0 || a->top_k <= 0 || a->x_row_stride % 8 != 0 ||
        (reinterpret_cast<uintptr_t>(a->x) & 15) || a->y_row_stride % 4 != 0 ||
        (reinterpret_cast<uintptr_t>(a->y) & 7))
        return NVMOE_ERR_INVALID_ARG;
    if (a->kernel < NVMOE_KERNEL_DEFAULT || a->kernel > NVMOE_KERNEL_F16)
        return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok == 0) return NVMOE_OK;
    if (prefill_use_fp4(a)) return prefill_fp4_run(a, (cudaStream_t)stream);
    PfParams P{};
    P.pool = pool;
    P.has_shared = a->shared ? 1 : 0;
    P.shared = a->shared ? *a->shared : pool;
    P.shared_gate = a->shared ? a->shared_gate : nullptr;
    P.x = a->x;
    P.x_stride = a->x_row_stride;
    P.ids = a->slot_ids;
    P.ids_stride = a->ids_row_stride;
    P.w = a->weights;
    P.w_stride = a->weights_row_stride;
    P.top_k = a->top_k;
    P.n_tok = a->n_tok;
    P.y = a->y;
    P.y_stride = a->y_row_stride;
    P.L = pf_layout(a->n_tok, a->top_k, H, I, pool.n_slots);
    P.status = a->status;
    if (!a->workspace || a->workspace_bytes < P.L.total ||
        (reinterpret_cast<uintptr_t>(a->workspace) & 255))
        return NVMOE_ERR_WORKSPACE;
    P.ws = static_cast<unsigned char*>(a->workspace);
    cudaStream_t st = (cudaStream_t)stream;
    // header (tile / entry counts, status) and the per-key counts start at zero
    NVMOE_CUDA_TRY(cudaMemsetAsync(P.ws + P.L.hdr, 0, P.L.base - P.L.hdr, st));
    const int n_sel = a->n_tok * a->top_k;
    const int gb = std::min(4 * kNumSMs, (n_sel + 255) / 256);
    pf_count<<<std::max(gb, 1), 256, 0, st>>>(P);
    pf_scan<<<1, 1024, 0, st>>>(P);
    const int n_all = a->n_tok * (a->top_k + 1);
    pf_scatter<<<std::min(4 * kNumSMs, (n_all + 255) / 256), 256, 0, st>>>(P);
    pf_gather<<<P.L.n_ent_max, 128, 0, st>>>(P);
    const int gu_smem = kStages * kGuStage, dn_smem = kStages * kDnStage;
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(pf_gate_up, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        gu_smem));
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(pf_down, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        dn_smem));
    pf_gate_up<<<dim3(P.L.max_tiles, I / kTileM, kTileN / kGuN), kPfThreads, gu_smem, st>>>(P);
    pf_down<<<dim3(P.L.max_tiles, H / kTileM), kPfThreads, dn_smem, st>>>(P);
    const int64_t n4 = (int64_t)a->n_tok * (H / 4);
    pf_combine<<<(int)std::min<int64_t>(8 * kNumSMs, (n4 + 255) / 256), 256, 0, st>>>(P);
    pf_status<<<1, 1, 0, st>>>(P);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}
