// R10 prefill on the block-scaled FP4 tensor cores: the routed-expert FFN for large batches as a
// token-sorted grouped GEMM of tcgen05.mma kind::mxf4nvf4 (E2M1 x E2M1, one UE4M3 scale per 16
// on both operands, fp32 accumulators in tensor memory).  The weights go from the slot banks to
// shared memory by TMA (128-byte swizzle) and into the MMA unchanged; the activations enter as
// kNT = 3 NVFP4 residual terms per row (about bf16 precision: each term quantises what the
// earlier ones left, two lanes per 16-block), so the result matches the f16 path and the oracle
// within the FFN tolerance.
//
// Same contract as nvmoe_moe_ffn_prefill's f16 path (nvme_offload_cache.py:1957-2013; llama.cpp
// mul_mat_id for n_tokens > 1, scripts/moe_cache_probe.cpp:1668-1684):
//   y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] )  (+ the shared expert).
// Steps (one stream, kernel boundaries order them):
//   count / scan / scatter — entries sorted by key (slot, or the shared expert), tiles of <= 42
//                            entries per key, each entry's (tile, row)
//   quant_x  — per token: the row exponent, the shared gate, then each K stage as 3 NVFP4 terms
//              into the gate_up B image of every tile row that holds the token
//   gate_up  — persistent: units (tile, 128-row j-block), gate and up blocks of M = 128 against
//              one B image, N = 3 x entries, K = H; epilogue h = silu(gate) * up (fp32)
//   act      — per entry: h row exponent, its K stages as NVFP4 terms into the down B image
//   down     — persistent: units (tile, 256 rows of H as two M = 128 blocks), K = I; epilogue
//              y_part[e] = w_e * row (fp32)
//   combine  — y[t] = sum over t's entries in the order j = 0..k (shared last) (bf16)
// Deterministic: every output element is one MMA accumulation and fixed-order sums.
#include "common.cuh"
#include "ffn_common.cuh"
#include "fp4_common.cuh"
#include "umma.cuh"

#include <algorithm>
#include <cstdlib>
#include <cstring>

namespace nvmoe {
using namespace fp4;
namespace {

constexpr int kNT = 3;                     // NVFP4 terms per activation row: B rows kNT i + t
constexpr int kTT = 42;                    // entries per tile: B rows 3 x 42 = 126 of 128
constexpr int kImg = 128 * 144;            // one K stage of a tile image (128 code rows + scales)
// One ring stage (K = 256): two 128-row weight blocks A0, A1 (the MMAs of a stage share the
// tile's B image), the B image, then the A0 and A1 scales.
constexpr int kNSt = 4;
constexpr int kOffA1 = 16384;
constexpr int kOffBi = 32768;
constexpr int kOffAs = kOffBi + kImg;
constexpr int kStg = kOffAs + 4096;        // 55296, every byte of it arrives by TMA
static_assert(kStg % 1024 == 0, "stage layout");
constexpr int kEpiWarps = 8;               // two per TMEM lane quadrant, 21 entries each
// + 4 scale-factor warps, the producer, the MMA issuer and the unit-info warp
constexpr int kGThreads = 32 * (kEpiWarps + 7);
constexpr int kWSf = kEpiWarps, kWProd = kEpiWarps + 4, kWMma = kEpiWarps + 5, kWInfo = kEpiWarps + 6;
// What the epilogue needs of a unit, prepared ahead by the unit-info warp in a ring of kInfoN.
struct UnitInfo {
    int eb, nr;
    float ga, gb;       // global scales of the A0 and A1 blocks
    int eexp[kTT];      // per entry: the row exponent of its B rows
    float efac[kTT];    // per entry: router weight (x shared gate), down phase
};
constexpr int kInfoN = 4;
constexpr int kOffBar = kNSt * kStg;       // mbarriers
constexpr int kOffMisc = kOffBar + 32 * 8; // tmem base, abort
constexpr int kOffInfo = kOffMisc + 64;
constexpr int kGSmem = kOffInfo + kInfoN * (int)sizeof(UnitInfo) + 1024;
// tensor memory: D0 | D1 (128 columns each), then per stage 48 scale columns (A0, A1, B)
constexpr uint32_t kTmD = 0, kTmSF = 256, kTmCols = 512;
static_assert(kTmSF + 48 * kNSt <= kTmCols, "tensor memory");

enum { QH_N_TILES = 0, QH_N_ENT = 1, QH_STATUS = 2 };


__device__ __forceinline__ int pf4_npad(int nr) { return (kNT * nr + 7) & ~7; }  // MMA N

// ---- activation quantiser for the tile images: a warp quantises one K stage (256 values, 16
// blocks) of one row; lanes 2 blk and 2 blk + 1 hold values 8 hf .. 8 hf + 7 of block blk.
// kNT residual terms as in fp4_common.cuh: per term the block maximum, a UE4M3 scale rounded up
// (times 2^(ke + 2 t)), E2M1 round-to-nearest.  code[t] = this lane's 4 code bytes of term t,
// byte t of scw = the block's scale code of term t.
__device__ __forceinline__ void quant_pair_terms(float (&v)[8], int ke, uint32_t (&code)[kNT],
                                                 uint32_t& scw) {
    scw = 0;
#pragma unroll
    for (int t = 0; t < kNT; ++t) {
        float am = 0.f;
#pragma unroll
        for (int k = 0; k < 8; ++k) am = fmaxf(am, fabsf(v[k]));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        const float target = am * (1.0f / 6.0f) * fp4_exp2(ke + 2 * t);
        uint32_t c8 = e4m3_code(target);
        float sv = e4m3_value(c8);
        if (sv < target && c8 < 0x7eu) sv = e4m3_value(++c8);  // round the scale up
        const float sc = sv * fp4_exp2(-(ke + 2 * t));
        const float inv = sc > 0.f ? 1.0f / sc : 0.f;
        uint32_t w;
        asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
            "mov.b32 %0, {b0, b1, b2, b3}; }"
            : "=r"(w)
            : "f"(v[0] * inv), "f"(v[1] * inv), "f"(v[2] * inv), "f"(v[3] * inv),
              "f"(v[4] * inv), "f"(v[5] * inv), "f"(v[6] * inv), "f"(v[7] * inv));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t h2 = e2m1x2_to_f16x2((uint16_t)((w >> (8 * j)) & 0xffu));
            const float2 d = __half22float2(*reinterpret_cast<const __half2*>(&h2));
            v[2 * j] = fmaf(-d.x, sc, v[2 * j]);
            v[2 * j + 1] = fmaf(-d.y, sc, v[2 * j + 1]);
        }
        code[t] = w;
        scw |= c8 << (8 * t);
    }
}
// Lane 4 t + L (t < kNT) collects the term-t scale codes of blocks 4 L .. 4 L + 3.
__device__ __forceinline__ uint32_t gather_scales(uint32_t scw) {
    const int lane = threadIdx.x & 31, t = (lane >> 2) & 3, L = lane & 3;
    uint32_t g = 0;
#pragma unroll
    for (int m = 0; m < 4; ++m) {
        const uint32_t w = __shfl_sync(0xffffffffu, scw, 2 * (4 * L + m));
        g |= ((w >> (8 * t)) & 0xffu) << (8 * m);
    }
    return g;
}
// Rows kNT i + t of one stage of a tile image (128 rows, 128-byte swizzle, scales after the code
// rows): each term row is one full 128-byte line (a 4-byte store per lane); the kNT rows' scale
// records are 16 kNT contiguous bytes, lanes 4 t + L store 4 each.
__device__ __forceinline__ void put_pair_rows(uint8_t* img, int i, const uint32_t (&code)[kNT],
                                              uint32_t gsc) {
    const int lane = threadIdx.x & 31, blk = lane >> 1, hf = lane & 1;
#pragma unroll
    for (int t = 0; t < kNT; ++t) {
        const int n = kNT * i + t;
        *reinterpret_cast<uint32_t*>(img + n * 128 + (((blk >> 1) ^ (n & 7)) << 4) + ((blk & 1) << 3) + 4 * hf) = code[t];
    }
    if (lane < 4 * kNT) *reinterpret_cast<uint32_t*>(img + 128 * 128 + kNT * i * 16 + 4 * lane) = gsc;
}

struct Pf4Layout {
    size_t hdr, cnt, base, cursor, tile_base, tiles, ent_tok, ent_w, ent_of, ent_pos, ent_xk,
        ent_fac, hk, ximg, himg, h32, ypart, total;
    int n_keys, n_ent_max, max_tiles, ksg, ksd;
};

__host__ __device__ inline Pf4Layout pf4_layout(int n_tok, int top_k, int H, int I, int n_slots) {
    Pf4Layout L;
    L.n_keys = n_slots + 1;  // the shared expert is key n_slots
    L.n_ent_max = n_tok * (top_k + 1);
    L.max_tiles = (L.n_ent_max + kTT - 1) / kTT + std::min(L.n_keys, L.n_ent_max);
    L.ksg = H / 256;
    L.ksd = I / 256;
    size_t o = 0;
    auto take = [&](size_t bytes) {
        const size_t at = o;
        o = align_up(o + bytes, 1024);
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
    L.ent_pos = take(4 * (size_t)L.n_ent_max);  // tile << 8 | row
    L.ent_xk = take(4 * (size_t)L.n_ent_max);   // the entry's token row exponent
    L.ent_fac = take(4 * (size_t)L.n_ent_max);  // router weight (x shared gate)
    L.hk = take(4 * (size_t)L.n_ent_max);
    L.ximg = take((size_t)L.max_tiles * L.ksg * kImg);
    L.himg = take((size_t)L.max_tiles * L.ksd * kImg);
    L.h32 = take(4 * (size_t)L.n_ent_max * I);
    L.ypart = take(2 * (size_t)L.n_ent_max * H);  // bf16 per-entry partials
    L.total = o;
    return L;
}

struct __align__(64) Pf4Params {
    CUtensorMap map[12];  // [routed pool, shared pool][the six maps of fp4_pool_maps]
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
    Pf4Layout L;
    int32_t* status;
};

template <typename T>
__device__ __forceinline__ T* qws(const Pf4Params& P, size_t off) {
    return reinterpret_cast<T*>(P.ws + off);
}

// ------------------------------------------------------------------ grouping
__global__ void pf4_count(const __grid_constant__ Pf4Params P) {
    const int n = P.n_tok * P.top_k, S = P.pool.n_slots;
    int* cnt = qws<int>(P, P.L.cnt);
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const int t = p / P.top_k, j = p - t * P.top_k;
        const int s = P.ids[(int64_t)t * P.ids_stride + j];
        const bool ok = s >= 0 && s < S;
        const unsigned same = __match_any_sync(__activemask(), ok ? s : -1);
        if (ok && (threadIdx.x & 31) == __ffs(same) - 1) atomicAdd(&cnt[s], __popc(same));
        if (s >= S) atomicExch(qws<int>(P, P.L.hdr) + QH_STATUS, NVMOE_ERR_BAD_SLOT);
    }
}

// One block: entry bases (exclusive scan over keys) and the tile list.
__global__ void __launch_bounds__(1024) pf4_scan(const __grid_constant__ Pf4Params P) {
    __shared__ int warp_sums[33];
    const int K = P.L.n_keys, S = P.pool.n_slots, tid = threadIdx.x;
    int* cnt = qws<int>(P, P.L.cnt);
    int* base = qws<int>(P, P.L.base);
    int* cursor = qws<int>(P, P.L.cursor);
    int* tile_base = qws<int>(P, P.L.tile_base);
    int* tiles = qws<int>(P, P.L.tiles);
    if (tid == 0) cnt[S] = P.has_shared ? P.n_tok : 0;
    __syncthreads();
    int run_e = 0, run_t = 0;
    for (int b0 = 0; b0 < K; b0 += blockDim.x) {
        const int s = b0 + tid;
        const int c = s < K ? cnt[s] : 0;
        const int nt = (c + kTT - 1) / kTT;
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
                tl[1] = run_e + re + i * kTT;
                tl[2] = min(kTT, c - i * kTT);
            }
        }
        run_e += tot_e;
        run_t += tot_t;
    }
    if (tid == 0) {
        int* hdr = qws<int>(P, P.L.hdr);
        hdr[QH_N_TILES] = run_t;
        hdr[QH_N_ENT] = run_e;
    }
}

__global__ void pf4_scatter(const __grid_constant__ Pf4Params P) {
    const int S = P.pool.n_slots, K1 = P.top_k + 1;
    int* cursor = qws<int>(P, P.L.cursor);
    const int* base = qws<int>(P, P.L.base);
    const int* tile_base = qws<int>(P, P.L.tile_base);
    int* ent_tok = qws<int>(P, P.L.ent_tok);
    float* ent_w = qws<float>(P, P.L.ent_w);
    int* ent_of = qws<int>(P, P.L.ent_of);
    int* ent_pos = qws<int>(P, P.L.ent_pos);
    const int n = P.n_tok * K1;
    for (int p = blockIdx.x * blockDim.x + threadIdx.x; p < n; p += gridDim.x * blockDim.x) {
        const int t = p / K1, j = p - t * K1;
        int e = -1, key = -1;
        if (j < P.top_k) {
            const int s = P.ids[(int64_t)t * P.ids_stride + j];
            const bool ok = s >= 0 && s < S;
            // one atomic per distinct slot of the warp; the order of entries inside a key
            // changes no result
            const unsigned same = __match_any_sync(__activemask(), ok ? s : -1);
            const int lead = __ffs(same) - 1, ln = threadIdx.x & 31;
            int e0 = 0;
            if (ok && ln == lead) e0 = atomicAdd(&cursor[s], __popc(same));
            e0 = __shfl_sync(same, e0, lead);
            if (ok) {
                e = e0 + __popc(same & ((1u << ln) - 1u));
                key = s;
                ent_tok[e] = t;
                ent_w[e] = P.w[(int64_t)t * P.w_stride + j];
            }
        } else if (P.has_shared) {
            e = base[S] + t;
            key = S;
            ent_tok[e] = t;
            ent_w[e] = 1.0f;
        }
        if (e >= 0) {
            const int r = e - base[key];
            ent_pos[e] = ((tile_base[key] + r / kTT) << 8) | (r % kTT);
        }
        ent_of[p] = e;
    }
}

// One block of 128 threads per token: the row exponent and the shared gate, then each K stage
// (warp w: stages w, w + 4, ...) as kNT NVFP4 terms into the gate_up image row of every entry
// of the token.  The values stay in registers between the two passes; the entries' image
// positions sit in shared memory.
__global__ void __launch_bounds__(128) pf4_quant_x(const __grid_constant__ Pf4Params P) {
    __shared__ float red[8];
    __shared__ int epos[33];  // image position (tile << 8 | row) of each entry, -1: none
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int K1 = P.top_k + 1, KSG = P.L.ksg;  // KSG = H / 256 <= 32
    const uint16_t* xr = P.x + (int64_t)t * P.x_stride;
    int ent = -1;
    if (tid < K1) {
        ent = qws<int>(P, P.L.ent_of)[t * K1 + tid];
        epos[tid] = ent >= 0 ? qws<int>(P, P.L.ent_pos)[ent] : -1;
    }
    uint4 xv[8];
    float am = 0.f, dot = 0.f;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int st = warp + 4 * m;
        xv[m] = make_uint4(0u, 0u, 0u, 0u);
        if (st < KSG) {
            const int off = 256 * st + 8 * lane;
            xv[m] = *reinterpret_cast<const uint4*>(xr + off);
            const uint32_t w4[4] = {xv[m].x, xv[m].y, xv[m].z, xv[m].w};
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = __uint_as_float(k & 1 ? w4[k >> 1] & 0xffff0000u : w4[k >> 1] << 16);
                am = fmaxf(am, fabsf(f));
                if (P.shared_gate) dot = fmaf(f, bf16_bits_to_f32(P.shared_gate[off + k]), dot);
            }
        }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
        dot += __shfl_xor_sync(0xffffffffu, dot, o);
    }
    if (lane == 0) red[warp] = am, red[4 + warp] = dot;
    __syncthreads();
    const int ke = fp4_row_exp(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])));
    if (ent >= 0) {
        float f = qws<float>(P, P.L.ent_w)[ent];
        if (tid == P.top_k && P.shared_gate)
            f *= 1.0f / (1.0f + expf(-(red[4] + red[5] + red[6] + red[7])));
        qws<int>(P, P.L.ent_xk)[ent] = ke;
        qws<float>(P, P.L.ent_fac)[ent] = f;
    }
    uint8_t* ximg = P.ws + P.L.ximg;
#pragma unroll
    for (int m = 0; m < 8; ++m) {
        const int st = warp + 4 * m;
        if (st >= KSG) break;
        const uint32_t w4[4] = {xv[m].x, xv[m].y, xv[m].z, xv[m].w};
        float v[8];
#pragma unroll
        for (int k = 0; k < 8; ++k)
            v[k] = __uint_as_float(k & 1 ? w4[k >> 1] & 0xffff0000u : w4[k >> 1] << 16);
        uint32_t code[kNT], scw;
        quant_pair_terms(v, ke, code, scw);
        const uint32_t gsc = gather_scales(scw);
        for (int j = 0; j < K1; ++j) {
            const int pos = epos[j];
            if (pos < 0) continue;
            put_pair_rows(ximg + ((int64_t)(pos >> 8) * KSG + st) * kImg, pos & 0xff, code, gsc);
        }
    }
}

// One warp per entry (8 per block): the h row's exponent, then each K stage of the row as kNT
// NVFP4 terms into the entry's row of the down image (lane l: values 256 s + 8 l .. + 8).
constexpr int kActWarps = 8;
template <int NS>  // I / 256
__global__ void __launch_bounds__(32 * kActWarps) pf4_act(const __grid_constant__ Pf4Params P) {
    const int e = blockIdx.x * kActWarps + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (e >= qws<int>(P, P.L.hdr)[QH_N_ENT]) return;  // the whole warp: the quantiser shuffles
    const float* hrow = qws<float>(P, P.L.h32) + (int64_t)e * (256 * NS);
    float4 hv[2 * NS];
    float am = 0.f;
#pragma unroll
    for (int m = 0; m < 2 * NS; ++m) {
        hv[m] = *reinterpret_cast<const float4*>(hrow + 256 * (m >> 1) + 8 * lane + 4 * (m & 1));
        am = fmaxf(am, fmaxf(fmaxf(fabsf(hv[m].x), fabsf(hv[m].y)), fmaxf(fabsf(hv[m].z), fabsf(hv[m].w))));
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
    const int kh = fp4_row_exp(am);
    if (lane == 0) qws<int>(P, P.L.hk)[e] = kh;
    const int pos = qws<int>(P, P.L.ent_pos)[e];
    uint8_t* himg = P.ws + P.L.himg;
#pragma unroll
    for (int s = 0; s < NS; ++s) {
        float v[8] = {hv[2 * s].x, hv[2 * s].y, hv[2 * s].z, hv[2 * s].w,
                      hv[2 * s + 1].x, hv[2 * s + 1].y, hv[2 * s + 1].z, hv[2 * s + 1].w};
        uint32_t code[kNT], scw;
        quant_pair_terms(v, kh, code, scw);
        put_pair_rows(himg + ((int64_t)(pos >> 8) * NS + s) * kImg, pos & 0xff, code, gather_scales(scw));
    }
}

// ------------------------------------------------------------------ the grouped GEMMs
// Persistent, one CTA per SM; units dealt round-robin (u = c, c + G, ...), so the units of one
// tile, and the tiles of one expert, run side by side and share their loads in L2.  A unit is
// two 128-row weight blocks against one tile: PH = 0 (gate_up) the gate and the up rows of a
// 128-row j-block, so one thread holds gate and up of the same j; PH = 1 (down) 256 rows of H.
// Warps 0-7 epilogue (two per TMEM lane quadrant, 16 entries each), 8-11 scale factors, 12
// producer (TMA weights + the tile's B image stage), 13 MMA issuer.  One D buffer: the MMAs of
// the next unit start when the epilogue has read D out, while the ring keeps loading.
template <int PH>
__global__ void __launch_bounds__(kGThreads, 1) pf4_gemm(const __grid_constant__ Pf4Params P) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* full = reinterpret_cast<uint64_t*>(sm + kOffBar);
    uint64_t* sf_full = full + kNSt;
    uint64_t* empty = full + 2 * kNSt;
    uint64_t* d_full = full + 3 * kNSt;
    uint64_t* d_empty = d_full + 1;
    uint64_t* info_full = d_full + 2;
    uint64_t* info_empty = info_full + kInfoN;
    uint32_t* tmem_p = reinterpret_cast<uint32_t*>(sm + kOffMisc);
    volatile int* abort = reinterpret_cast<int*>(sm + kOffMisc) + 1;
    UnitInfo* info = reinterpret_cast<UnitInfo*>(sm + kOffInfo);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int H = P.pool.hidden, I = P.pool.inter, S = P.pool.n_slots;
    const int UPT = PH ? H / 256 : I / 128;  // units per tile
    const int KS = PH ? P.L.ksd : P.L.ksg;   // K stages per unit

    if (tid == 0) {
        for (int s = 0; s < kNSt; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&sf_full[s], 4);
            mbar_init(&empty[s], 1);
        }
        mbar_init(d_full, 1);
        mbar_init(d_empty, kEpiWarps);
        for (int b = 0; b < kInfoN; ++b) {
            mbar_init(&info_full[b], 1);
            mbar_init(&info_empty[b], kEpiWarps);
        }
        *abort = 0;
        mbar_init_fence();
    }
    if (warp == kWMma) umma::tmem_alloc(tmem_p, kTmCols);
    if (warp == kWProd && lane < 12) prefetch_map(&P.map[lane]);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tm = *tmem_p;

    const int n_tiles = qws<int>(P, P.L.hdr)[QH_N_TILES];
    const int* tiles = qws<int>(P, P.L.tiles);
    const int n_units = n_tiles * UPT;
    const int my_units = n_units > c ? (n_units - 1 - c) / G + 1 : 0;
    const uint8_t* img = P.ws + (PH ? P.L.himg : P.L.ximg);
    bool ok = true;

    if (warp == kWProd) {
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int it = 0;
            int key_next = my_units > 0 ? tiles[3 * (c / UPT)] : 0;
            for (int k = 0; k < my_units && ok; ++k) {
                const int u = c + k * G, tile = u / UPT, sub = u - tile * UPT;
                const int key = key_next;
                if (k + 1 < my_units) key_next = tiles[3 * ((u + G) / UPT)];
                const bool sh = key == S;
                const int slot = sh ? 0 : key;
                const CUtensorMap* m = P.map + (sh ? 6 : 0);
                for (int ks = 0; ks < KS; ++ks, ++it) {
                    const int s = it % kNSt;
                    if (it >= kNSt && !wait_bar(&empty[s], ((it / kNSt) + 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = sm + s * kStg;
                    mbar_arrive_expect_tx(&full[s], kStg);
                    if (PH == 0) {  // gate and up boxes are 64 rows: two per block
                        const int y = sub * 128;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            tma_load_3d(st + 8192 * h, m + M_GATE, ks * 128, y + 64 * h, slot, &full[s], pol);
                            tma_load_3d(st + kOffA1 + 8192 * h, m + M_UP, ks * 128, y + 64 * h, slot, &full[s], pol);
                            tma_load_3d(st + kOffAs + 1024 * h, m + M_GATE_SF, ks * 16, y + 64 * h, slot, &full[s], pol);
                            tma_load_3d(st + kOffAs + 2048 + 1024 * h, m + M_UP_SF, ks * 16, y + 64 * h, slot, &full[s], pol);
                        }
                    } else {
                        const int y = sub * 256;
#pragma unroll
                        for (int h = 0; h < 2; ++h) {
                            tma_load_3d(st + kOffA1 * h, m + M_DOWN, ks * 128, y + 128 * h, slot, &full[s], pol);
                            tma_load_3d(st + kOffAs + 2048 * h, m + M_DOWN_SF, ks * 16, y + 128 * h, slot, &full[s], pol);
                        }
                    }
                    bulk_g2s(st + kOffBi, img + ((int64_t)tile * KS + ks) * kImg, kImg, &full[s]);
                }
            }
            if (!ok) {
                for (int k = std::max(0, it - kNSt); k < it; ++k)
                    mbar_wait_bounded(&full[k % kNSt], (k / kNSt) & 1, 1u << 16);
            }
        }
        __syncwarp();
    } else if (warp == kWMma) {
        int it = 0;
        int nr_next = my_units > 0 ? tiles[3 * (c / UPT) + 2] : 0;
        for (int k = 0; k < my_units && ok; ++k) {
            const int u = c + k * G;
            const int nr = nr_next;
            if (k + 1 < my_units) nr_next = tiles[3 * ((u + G) / UPT) + 2];
            const uint32_t idesc = umma::idesc_mxf4(128, pf4_npad(nr));
            if (k >= 1 && !wait_bar(d_empty, (k - 1) & 1, abort)) {
                ok = false;
                break;
            }
            umma::fence_after_sync();
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % kNSt;
                if (!wait_bar(&sf_full[s], (it / kNSt) & 1, abort)) {
                    ok = false;
                    break;
                }
                umma::fence_after_sync();
                if (lane == 0) {
                    const uint32_t sa = smem_u32(sm + s * kStg);
                    const uint32_t sf = tm + kTmSF + 48 * s;
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const uint32_t acc = (ks == 0 && i == 0) ? 0u : 1u;
                        const uint64_t bd = umma::smem_desc_sw128(sa + kOffBi + 32 * i);
                        umma::mma_mxf4(tm + kTmD, umma::smem_desc_sw128(sa + 32 * i), bd, idesc,
                                       sf + 4 * i, sf + 32 + 4 * i, acc);
                        umma::mma_mxf4(tm + kTmD + 128, umma::smem_desc_sw128(sa + kOffA1 + 32 * i),
                                       bd, idesc, sf + 16 + 4 * i, sf + 32 + 4 * i, acc);
                    }
                    umma::commit(&empty[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) umma::commit(d_full);
            __syncwarp();
        }
    } else if (warp == kWInfo) {
        const int* ent_xk = qws<int>(P, P.L.ent_xk);
        const float* ent_fac = qws<float>(P, P.L.ent_fac);
        const int* hk = qws<int>(P, P.L.hk);
        int4 tn = make_int4(0, 0, 0, 0);  // the next unit's tile record
        if (my_units > 0) tn = make_int4(tiles[3 * (c / UPT)], tiles[3 * (c / UPT) + 1], tiles[3 * (c / UPT) + 2], 0);
        for (int k = 0; k < my_units && ok; ++k) {
            const int b = k % kInfoN, u = c + k * G;
            const int key = tn.x, eb = tn.y, nr = tn.z;
            if (k + 1 < my_units) {
                const int t1 = (u + G) / UPT;
                tn = make_int4(tiles[3 * t1], tiles[3 * t1 + 1], tiles[3 * t1 + 2], 0);
            }
            const bool sh = key == S;
            const nvmoe_expert_pool& pool = sh ? P.shared : P.pool;
            const int slot = sh ? 0 : key;
            int ex[2] = {0, 0};
            float fa[2] = {0.f, 0.f};
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int i = lane + 32 * h;
                if (i < nr) {
                    ex[h] = PH ? hk[eb + i] : ent_xk[eb + i];
                    if (PH) fa[h] = ent_fac[eb + i];
                }
            }
            const float ga = global_of(PH ? pool.down : pool.gate, slot);
            const float gb = PH ? ga : global_of(pool.up, slot);
            if (k >= kInfoN && !wait_bar(&info_empty[b], ((k / kInfoN) + 1) & 1, abort)) {
                ok = false;
                break;
            }
            UnitInfo& in = info[b];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                if (lane + 32 * h < kTT) {
                    in.eexp[lane + 32 * h] = ex[h];
                    in.efac[lane + 32 * h] = fa[h];
                }
            }
            if (lane == 0) in.eb = eb, in.nr = nr, in.ga = ga, in.gb = gb;
            __syncwarp();
            if (lane == 0) mbar_arrive(&info_full[b]);
        }
    } else if (warp >= kWSf) {
        // scale factors of A0, A1 and B, 128 rows each -> column 4 i + r / 32, lane r % 32 of
        // every quadrant
        const int qd = warp & 3;
        int it = 0;
        for (int k = 0; k < my_units && ok; ++k) {
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % kNSt;
                if (!wait_bar(&full[s], (it / kNSt) & 1, abort)) {
                    ok = false;
                    break;
                }
                const uint8_t* st = sm + s * kStg;
                uint32_t va0[16], va1[16], vb[16];
#pragma unroll
                for (int m1 = 0; m1 < 4; ++m1) {
                    const int row = 32 * m1 + lane;
                    const uint4 a0 = *reinterpret_cast<const uint4*>(st + kOffAs + row * 16);
                    const uint4 a1 = *reinterpret_cast<const uint4*>(st + kOffAs + 2048 + row * 16);
                    const uint4 b = *reinterpret_cast<const uint4*>(st + kOffBi + 128 * 128 + row * 16);
                    va0[m1] = a0.x, va0[4 + m1] = a0.y, va0[8 + m1] = a0.z, va0[12 + m1] = a0.w;
                    va1[m1] = a1.x, va1[4 + m1] = a1.y, va1[8 + m1] = a1.z, va1[12 + m1] = a1.w;
                    vb[m1] = b.x, vb[4 + m1] = b.y, vb[8 + m1] = b.z, vb[12 + m1] = b.w;
                }
                const uint32_t ta = tm + ((uint32_t)(qd * 32) << 16) + kTmSF + 48 * s;
                umma::st_x16(ta, va0);
                umma::st_x16(ta + 16, va1);
                umma::st_x16(ta + 32, vb);
                umma::wait_st();
                umma::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&sf_full[s]);
            }
        }
    } else {
        // epilogue: row r of the unit's two D blocks (the same weight row index in A0 and A1),
        // entries 16 hh .. 16 hh + 15 (a column group of 4 terms each)
        const int r = 32 * (warp & 3) + lane, hh = warp >> 2, i0 = 16 * hh;
        float* h32 = qws<float>(P, P.L.h32);
        uint16_t* ypart = qws<uint16_t>(P, P.L.ypart);
        for (int k = 0; k < my_units && ok; ++k) {
            const int b = k % kInfoN, u = c + k * G, sub = u % UPT;
            if (!wait_bar(&info_full[b], (k / kInfoN) & 1, abort)) {
                ok = false;
                break;
            }
            const UnitInfo& in = info[b];
            const int eb = in.eb, nr = in.nr;
            const float ga = in.ga, gb = in.gb;
            if (!wait_bar(d_full, k & 1, abort)) {
                ok = false;
                break;
            }
            umma::fence_after_sync();
            // Columns 3 e + t.  Half hh reads its own group of 16 entries (columns 48 hh ..
            // 48 hh + 47) and the last group (entries 32..41, columns 96..125), whose entries
            // 32 + 5 hh .. + 4 it stores.
            float g0[16], g1[16], x0[10], x1[10];
#pragma unroll
            for (int i = 0; i < 16; ++i) g0[i] = g1[i] = 0.f;
#pragma unroll
            for (int i = 0; i < 10; ++i) x0[i] = x1[i] = 0.f;
#pragma unroll
            for (int ch = 0; ch < 5; ++ch) {
                const int cl = ch < 3 ? ch : ch - 3;  // chunk within its group
                const int cb = ch < 3 ? 48 * hh + 16 * cl : 96 + 16 * cl;
                if ((ch < 3 ? i0 : 32) + (16 * cl) / 3 >= nr) continue;
                uint32_t d0[16], d1[16];
                umma::ld_x16(umma::lane_addr(tm, warp, kTmD + cb), d0);
                umma::ld_x16(umma::lane_addr(tm, warp, kTmD + 128 + cb), d1);
                umma::wait_ld();
#pragma unroll
                for (int j = 0; j < 16; ++j) {
                    const int col = 16 * cl + j, le = col / 3;
                    const float f = fp4_exp2(-2 * (col % 3));
                    if (ch < 3) {
                        g0[le] = fmaf(__uint_as_float(d0[j]), f, g0[le]);
                        g1[le] = fmaf(__uint_as_float(d1[j]), f, g1[le]);
                    } else if (le < 10) {
                        x0[le] = fmaf(__uint_as_float(d0[j]), f, x0[le]);
                        x1[le] = fmaf(__uint_as_float(d1[j]), f, x1[le]);
                    }
                }
            }
            umma::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(d_empty);
            auto emit = [&](int e, float a, float bb) {
                if (PH == 0) {
                    const float f = fp4_exp2(-in.eexp[e]);
                    h32[(int64_t)(eb + e) * I + sub * 128 + r] = silu(a * f * ga) * (bb * f * gb);
                } else {
                    const float f = fp4_exp2(-in.eexp[e]) * in.efac[e] * ga;
                    // (bf16 partials: half the bytes of the largest write and read of the
                    // layer; each is within 2^-9 of the fp32 partial, and the sum and the
                    // output rounding stay as before)
                    uint16_t* yp = ypart + (int64_t)(eb + e) * H + sub * 256 + r;
                    yp[0] = f32_to_bf16_bits(a * f);
                    yp[128] = f32_to_bf16_bits(bb * f);
                }
            };
#pragma unroll
            for (int i = 0; i < 16; ++i)
                if (i0 + i < nr) emit(i0 + i, g0[i], g1[i]);
#pragma unroll
            for (int i = 0; i < 10; ++i)
                if (i / 5 == hh && 32 + i < nr) emit(32 + i, x0[i], x1[i]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&info_empty[b]);
        }
    }
    if (!ok && tid % 32 == 0) atomicExch(qws<int>(P, P.L.hdr) + QH_STATUS, NVMOE_ERR_TIMEOUT);

    umma::fence_before_sync();
    __syncthreads();
    if (warp == kWMma) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tm, kTmCols);
    }
}

// y[t] = sum_j y_part[ent_of[t, j]] (bf16 partials, fp32 sum) in the order j = 0..k-1, shared;
// 4 columns per thread.
__global__ void pf4_combine(const __grid_constant__ Pf4Params P) {
    const int H = P.pool.hidden, K1 = P.top_k + 1;
    const int* ent_of = qws<int>(P, P.L.ent_of);
    const uint16_t* yp = qws<uint16_t>(P, P.L.ypart);
    const int64_t n4 = (int64_t)P.n_tok * (H / 4);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n4;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (H / 4)), cc = (int)(i % (H / 4)) * 4;
        float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int j = 0; j < K1; ++j) {
            const int e = ent_of[t * K1 + j];
            if (e < 0) continue;
            const uint2 v = *reinterpret_cast<const uint2*>(yp + (int64_t)e * H + cc);
            s.x += __uint_as_float(v.x << 16), s.y += __uint_as_float(v.x & 0xffff0000u);
            s.z += __uint_as_float(v.y << 16), s.w += __uint_as_float(v.y & 0xffff0000u);
        }
        uint2 o;
        o.x = (uint32_t)f32_to_bf16_bits(s.x) | ((uint32_t)f32_to_bf16_bits(s.y) << 16);
        o.y = (uint32_t)f32_to_bf16_bits(s.z) | ((uint32_t)f32_to_bf16_bits(s.w) << 16);
        *reinterpret_cast<uint2*>(P.y + (int64_t)t * P.y_stride + cc) = o;
    }
}

__global__ void pf4_status(const __grid_constant__ Pf4Params P) {
    if (P.status) *P.status = qws<int>(P, P.L.hdr)[QH_STATUS];
}

}  // namespace

// Shapes and banks the FP4 prefill covers (NVFP4, H a multiple of 512 up to 8192, I of 256 up to 1536,
// every bank usable by TMA).
bool prefill_fp4_ok(const nvmoe_ffn_args* a) {
    const nvmoe_expert_pool& p = *a->pool;
    if (p.quant != NVMOE_Q_NVFP4 || p.hidden % 512 != 0 || p.hidden > 8192 || p.inter % 256 != 0 ||
        p.inter > 1536 || a->top_k > 32)
        return false;
    CUtensorMap m[6];
    if (!fp4_pool_maps(p, m)) return false;
    if (a->shared && !fp4_pool_maps(*a->shared, m)) return false;
    return true;
}

size_t prefill_fp4_workspace(int n_tok, int top_k, int H, int I, int n_slots) {
    return pf4_layout(std::max(n_tok, 1), top_k, H, I, n_slots).total;
}

// Validated arguments (the caller checked pointers, alignment and shapes).
int prefill_fp4_run(const nvmoe_ffn_args* a, cudaStream_t st) {
    Pf4Params P;
    std::memset(&P, 0, sizeof(P));
    const nvmoe_expert_pool& pool = *a->pool;
    if (!fp4_pool_maps(pool, P.map)) return NVMOE_ERR_UNSUPPORTED;
    if (!fp4_pool_maps(a->shared ? *a->shared : pool, P.map + 6)) return NVMOE_ERR_UNSUPPORTED;
    const int H = pool.hidden, I = pool.inter;
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
    P.L = pf4_layout(a->n_tok, a->top_k, H, I, pool.n_slots);
    P.status = a->status;
    if (!a->workspace || a->workspace_bytes < P.L.total ||
        (reinterpret_cast<uintptr_t>(a->workspace) & 255))
        return NVMOE_ERR_WORKSPACE;
    P.ws = static_cast<unsigned char*>(a->workspace);
    int dev = 0, sms = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    NVMOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    NVMOE_CUDA_TRY(cudaMemsetAsync(P.ws + P.L.hdr, 0, P.L.base - P.L.hdr, st));
    const int n_sel = a->n_tok * a->top_k;
    pf4_count<<<std::max(1, std::min(4 * sms, (n_sel + 255) / 256)), 256, 0, st>>>(P);
    pf4_scan<<<1, 1024, 0, st>>>(P);
    const int n_all = a->n_tok * (a->top_k + 1);
    pf4_scatter<<<std::max(1, std::min(4 * sms, (n_all + 255) / 256)), 256, 0, st>>>(P);
    pf4_quant_x<<<a->n_tok, 128, 0, st>>>(P);
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(pf4_gemm<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem));
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(pf4_gemm<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, kGSmem));
    pf4_gemm<0><<<sms, kGThreads, kGSmem, st>>>(P);
    const int act_blocks = (P.L.n_ent_max + kActWarps - 1) / kActWarps;
    switch (I / 256) {  // I is a multiple of 256 up to 1536
        case 1: pf4_act<1><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
        case 2: pf4_act<2><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
        case 3: pf4_act<3><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
        case 4: pf4_act<4><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
        case 5: pf4_act<5><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
        default: pf4_act<6><<<act_blocks, 32 * kActWarps, 0, st>>>(P); break;
    }
    pf4_gemm<1><<<sms, kGThreads, kGSmem, st>>>(P);
    const int64_t n4 = (int64_t)a->n_tok * (H / 4);
    pf4_combine<<<(int)std::min<int64_t>(8 * sms, (n4 + 255) / 256), 256, 0, st>>>(P);
    pf4_status<<<1, 1, 0, st>>>(P);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}

}  // namespace nvmoe
