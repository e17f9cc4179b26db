// NVFP4 expert FFN on the 5th-generation tensor cores (decode and small batches).
//
// The routed-expert FFN of one layer step,
//     y[t] = sum_j w[t,j] * down( silu(gate x[t]) * up x[t] )  (+ the shared expert),
// for NVFP4 slot pools, as block-scaled FP4 MMAs (tcgen05.mma kind::mxf4nvf4: E2M1 values with
// one UE4M3 scale per 16, fp32 accumulators in tensor memory).  The weights move from HBM to
// shared memory by TMA (128-byte swizzle, L2 evict-first) and feed the tensor core as stored in
// the slot banks: nothing is dequantised on the CUDA cores.  The pool's per-16 E4M3 scales are
// the A scale factors, its per-matrix fp32 scale is applied in the epilogue.
//
// Activations as FP4 terms.  The MMA takes both operands in NVFP4, so every activation row
// (x for gate/up, h for down) enters as a sum of kFp4Terms NVFP4 rows: term t quantises the
// residual left by terms 0..t-1 (E2M1 round-to-nearest, per-16 UE4M3 scale rounded up so the
// block fits).  Each row has a power-of-two exponent k from its maximum (|max| 2^k in
// [1024, 2048)) and term t's scales are stored times 2^(k + 2t), which keeps every term's scales
// in the E4M3 range for blocks down to ~2^-17 of the row maximum.  Each term is a separate B row
// (N = 4 x tokens) and the epilogue sums the term columns with their factors: with 4 terms the
// residual is below 2^-9 of each 16-block's maximum, under the bf16 rounding of the output.
//
// Work split (persistent grid, one CTA per SM).  A gate_up unit is (group, 64-row j-block): the
// MMA tile stacks gate rows [64 jb, 64 jb + 64) over the up rows of the same j (M = 128), so one
// CTA owns matching gate / up values; K = H in stages of 256.  A down unit is (group, 128-row
// block of H), K = I.  Units are never cut.  Gate_up units are dealt round-robin (unit u to CTA
// u mod G, numbered group-major), so each round of G units completes the next groups; down units
// go first to the CTAs with one gate_up unit fewer (they finish their round earlier and take the
// earliest groups), then in equal contiguous shares over all CTAs.
//
// Dataflow.  (0) Every CTA quantises a share of the (token, 16-block) activation jobs into
// per-token images (both swizzle phases a token can take in a group); the gate_up B rows of a
// group are gathered from them by 1-D bulk copies.  (1) A gate_up unit's epilogue computes
// h = silu(gate) * up in fp32 for its 64 j and every token of the group; the group's last unit
// to be stored (atomic count) quantises all of the group's h rows into its down image.  (2) A
// down unit's epilogue stores each entry's weighted rows.  (3) After a grid barrier every CTA
// sums its slice of y over each token's entries in the order j = 0..k (shared expert last).
// All cross-CTA handoffs are release / acquire counters with bounded waits; the sums are in a
// fixed order, so results are deterministic and do not depend on the grid size.
//
// Warp roles (352 threads): 0-3 epilogue (TMEM lane quadrants 0-3), 4-7 scale factors (pool
// scales and activation scales from shared memory into tensor memory), 8 weight TMA producer,
// 9 activation producer (waits on the image counters), 10 MMA issuer.  Warps 0-7 first
// quantise this CTA's share of the activation jobs.
//
// References: the FFN of one slot group follows nvme_offload_cache.py:1989-2135 (_expert_gemm /
// the shared expert at :2115-2123); the NVFP4 bank layout is the FTW layout
// (nvme_offload_cache.py:764-835, scripts/convert_ftw_to_gguf.py:54-58).
#include <cuda.h>  // CUtensorMap and its enums (the encoder itself comes through the runtime)

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "common.cuh"
#include "ffn_common.cuh"
#include "umma.cuh"
#include "fp4_common.cuh"

namespace nvmoe {
namespace {

constexpr int kNS = 8;                                // ring stages
constexpr int kThreads = 352;                         // 11 warps
constexpr int kOffB = 16384;                          // A codes [0, 16 KB), then the B image
constexpr int kOffASF = kOffB + kFp4ImgStage;         // A scales [128 rows][16 B]
constexpr int kStageBytes = 23552;                    // 1024-aligned stage
constexpr int kRing = kNS * kStageBytes;
constexpr int kMaxGroups = 512;                       // group tables kept in shared memory
constexpr int kMaxTok = 256;
constexpr int kMaxEntOf = 2048;                       // (token, k) entry map kept in shared memory
constexpr int kMaxK1 = 33;                            // top-k (<= 32) + the shared expert
// misc shared memory after the ring
constexpr int kOffBars = kRing;                                 // 48 mbarriers
constexpr int kOffMisc = kOffBars + 48 * 8;                     // tmem base, flags
constexpr int kOffGrp = kOffMisc + 256;                         // e0 / nt / slot+pool per group
constexpr int kOffXk = kOffGrp + 3 * 4 * kMaxGroups;            // x term exponent per token
constexpr int kOffSg = kOffXk + 4 * kMaxTok;                    // shared-expert gate per token
constexpr int kOffEnt = kOffSg + 4 * kMaxTok;                   // entry of (token, j)
constexpr int kOffEtok = kOffEnt + 4 * kMaxEntOf;               // token of each entry
constexpr int kOffX = kOffEtok + 4 * kMaxEntOf;                  // up values [64][8] fp32
constexpr int kSmemTotal = kOffX + 64 * 8 * 4 + 1024;            // + alignment slack
static_assert(kOffB % 1024 == 0 && kStageBytes % 1024 == 0, "swizzled tiles need 1 KB alignment");
static_assert(kOffASF + 2048 <= kStageBytes, "stage overflow");
static_assert(kSmemTotal <= 227 * 1024, "shared memory");
// tensor memory columns: kND D buffers of 32, then per-stage scale factors (4 MMAs, 4-column
// aligned).  Six D buffers let the MMAs run units ahead of an epilogue that is building h rows.
constexpr int kND = 6;
constexpr uint32_t kTmD = 0, kTmSFA = 32 * kND, kTmSFB = kTmSFA + 16 * kNS, kTmCols = 512;
static_assert(kTmSFB + 16 * kNS <= kTmCols, "tensor memory overflow");
// grid phase counters (workspace ints, zeroed by the kernel before this one)
enum { PH_X = 0, PH_DN = 1 };

// Term t of a row with exponent k is stored with its scales multiplied by 2^(k + 2 t): the row
// maximum lands in [1024, 2048) (term 0's largest scale near 256, under the E4M3 limit of 448)
// and each later term, whose residual is ~5x smaller, gains a factor 4, so every term's scales
// stay in the E4M3 normal range for blocks down to ~2^-17 of the row maximum.

struct __align__(64) Fp4Params {
    CUtensorMap map[12];  // [pool][gate codes, gate scales, up codes, up scales, down ...]
    FfnParams P;
};

__device__ __forceinline__ void report_status(const FfnParams& P, int code) {
    atomicExch(wsp<int>(P, P.L.hdr) + HDR_STATUS, code);
    if (P.status) atomicExch(P.status, code);
}
__device__ __forceinline__ void report_timeout(const FfnParams& P) {
    report_status(P, NVMOE_ERR_TIMEOUT);
}

using namespace fp4;

struct Smem {
    uint8_t* base;
    uint64_t* full;     // [kNS] two producers, with bytes
    uint64_t* sf_full;  // [kNS] the 4 scale warps
    uint64_t* empty;    // [kNS] MMA commit
    uint64_t* d_full;   // [kND]
    uint64_t* d_empty;  // [kND] the 4 epilogue warps
    uint32_t* tmem;
    int* abort;
    int* misc;          // [0] last j-block flag
    int* g_e0;
    int* g_nt;
    int* g_sp;          // slot | pool << 24
    int* xk;
    float* sg;
    int* ent;           // ent_of [n_tok][k + 1]
    int* etok;          // token of each entry
    float* xbuf;
};

__device__ __forceinline__ Smem carve(uint8_t* raw) {
    Smem S;
    S.base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(raw) + 1023) & ~(uintptr_t)1023);
    uint64_t* bars = reinterpret_cast<uint64_t*>(S.base + kOffBars);
    S.full = bars;
    S.sf_full = bars + kNS;
    S.empty = bars + 2 * kNS;
    S.d_full = bars + 3 * kNS;
    S.d_empty = bars + 3 * kNS + kND;
    int* misc = reinterpret_cast<int*>(S.base + kOffMisc);
    S.tmem = reinterpret_cast<uint32_t*>(misc);
    S.abort = misc + 1;
    S.misc = misc + 4;
    S.g_e0 = reinterpret_cast<int*>(S.base + kOffGrp);
    S.g_nt = S.g_e0 + kMaxGroups;
    S.g_sp = S.g_nt + kMaxGroups;
    S.xk = reinterpret_cast<int*>(S.base + kOffXk);
    S.sg = reinterpret_cast<float*>(S.base + kOffSg);
    S.ent = reinterpret_cast<int*>(S.base + kOffEnt);
    S.etok = reinterpret_cast<int*>(S.base + kOffEtok);
    S.xbuf = reinterpret_cast<float*>(S.base + kOffX);
    return S;
}

// The CTA's work, in order: gate_up units c, c + G, ... (whole units, group-major numbering
// u = g * JB + jb, so each round of G units completes the next groups), then down units
// (u = g * RB + rb) from up to two contiguous ranges.  Down units go first to the CTAs with
// one gate_up unit fewer (they finish their gate_up round earlier and take the earliest
// groups), as many as equalise the stage counts, the rest in equal contiguous shares over all
// CTAs.
struct WorkList {
    int n1;            // gate_up units
    int d0, d1, d2, d3;  // down ranges [d0, d1), [d2, d3)
    __device__ __forceinline__ int count() const { return n1 + (d1 - d0) + (d3 - d2); }
    // k-th unit: phase (0 gate_up, 1 down) and unit index
    __device__ __forceinline__ void at(int k, int c, int G, int& ph, int& u) const {
        if (k < n1) { ph = 0; u = c + k * G; return; }
        k -= n1;
        ph = 1;
        u = k < d1 - d0 ? d0 + k : d2 + (k - (d1 - d0));
    }
};
__device__ __forceinline__ WorkList work_list(int c, int G, int U1, int U2, int KSG, int KSD) {
    WorkList W;
    const int q = U1 / G, r = U1 % G;
    W.n1 = q + (c < r ? 1 : 0);
    W.d0 = W.d1 = W.d2 = W.d3 = 0;
    if (r == 0) {
        W.d2 = range_lo(U2, c, G), W.d3 = range_lo(U2, c + 1, G);
        return W;
    }
    const int fill = KSG / KSD > 0 ? KSG / KSD : 1;  // down units that equal one gate_up unit
    const int cap = (G - r) * fill;
    if (U2 <= cap) {
        if (c >= r) W.d0 = range_lo(U2, c - r, G - r), W.d1 = range_lo(U2, c - r + 1, G - r);
        return W;
    }
    if (c >= r) W.d0 = (c - r) * fill, W.d1 = (c - r + 1) * fill;
    W.d2 = cap + range_lo(U2 - cap, c, G), W.d3 = cap + range_lo(U2 - cap, c + 1, G);
    return W;
}

// ------------------------------------------------------------------ the kernel
__global__ void __launch_bounds__(kThreads, 1) ffn_fp4_kernel(const __grid_constant__ Fp4Params A) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    const FfnParams& P = A.P;
    const WsLayout& L = P.L;
    const Smem S = carve(smem_raw);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int c = blockIdx.x, G = gridDim.x;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int JB = L.jb, RB = L.rb, KSG = L.ks_gu, KSD = L.ks_dn;

    if (tid == 0) {
        for (int s = 0; s < kNS; ++s) {
            mbar_init(&S.full[s], 2);
            mbar_init(&S.sf_full[s], 4);
            mbar_init(&S.empty[s], 1);
        }
        for (int b = 0; b < kND; ++b) {
            mbar_init(&S.d_full[b], 1);
            mbar_init(&S.d_empty[b], 4);
        }
        *S.abort = 0;
        mbar_init_fence();
    }
    if (warp == 10) umma::tmem_alloc(S.tmem, kTmCols);
    if (warp == 8 && lane < 12) prefetch_map(&A.map[lane]);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tm = *S.tmem;

    // everything below reads what the kernels before this one wrote (records, x, counters)
    grid_dep_wait();
    grid_dep_launch();
    const int* hdr = wsp<int>(P, L.hdr);
    const int n_groups = __ldcg(hdr + HDR_N_GROUPS);
    const int n_ent = __ldcg(hdr + HDR_N_ENT);
    const int* desc = wsp<int>(P, L.grp_desc);
    const int K1 = P.top_k + 1, NE = P.n_tok * K1;
    const float* sgate = (P.has_shared && P.shared_gate) ? wsp<float>(P, L.sg) : nullptr;

    // ---- one round of loads into shared memory: group tables, entry map, exponents, gates
    // (read for every group / entry the workspace holds, in flight with the header read; the
    // unused tail is never looked at)
    for (int g = tid; g < L.g_max; g += kThreads) {
        const int* d = desc + (int64_t)g * kDescInts;
        S.g_e0[g] = __ldcg(d + GD_E0);
        S.g_nt[g] = __ldcg(d + GD_NT);
        S.g_sp[g] = __ldcg(d + GD_SLOT) | (__ldcg(d + GD_POOL) << 24);
    }
    {
        const int* ent_of = wsp<int>(P, L.ent_of);
        const int* ent_tok = wsp<int>(P, L.ent_tok);
        for (int i = tid; i < NE; i += kThreads) {
            S.ent[i] = __ldcg(ent_of + i);
            S.etok[i] = __ldcg(ent_tok + i);
        }
        for (int t = tid; t < P.n_tok; t += kThreads) {
            S.xk[t] = __ldcg(wsp<int>(P, L.xk) + t);
            S.sg[t] = sgate ? __ldcg(sgate + t) : 1.0f;
        }
    }
    if (n_groups <= 0 || n_groups > kMaxGroups) {
        // nothing routed (or an upstream error): y = 0
        for (int i = c * kThreads + tid; i < P.n_tok * H; i += G * kThreads) {
            const int t = i / H, col = i - t * H;
            P.y[(int64_t)t * P.y_stride + col] = 0;
        }
        if (n_groups > kMaxGroups && c == 0 && tid == 0) report_status(P, NVMOE_ERR_GROUP_LIMIT);
    }
    const int NG = (n_groups > 0 && n_groups <= kMaxGroups) ? n_groups : 0;
    const int U1 = NG * JB, U2 = NG * RB;
    const WorkList W = work_list(c, G, U1, U2, KSG, KSD);
    const int n_units = NG ? W.count() : 0;
    __syncthreads();

    uint8_t* bimg = P.ws + L.bimg;
    uint8_t* ximg = P.ws + L.ximg;                        // [token][ks][2 phases][512 B]
    uint8_t* xsf = ximg + (int64_t)P.n_tok * KSG * 1024;  // [token][ks][4 rows][16 B]
    int* phase = wsp<int>(P, L.phase);
    int* gcnt = wsp<int>(P, L.gcnt);  // [g][0]: gate_up units stored, [g][1]: h rows built
    volatile int* abort = S.abort;
    const int HB = H / 16;

    // ---- 0. this CTA's share of the (entry, 16-block) activation jobs: the token's 16 values
    // as NVFP4 terms in the gate_up image of the entry's group
    if (warp < 8 && NG) {
        // 4 lanes per job, 64 jobs per round of the 256 threads (rounds uniform per warp)
        const int J = P.n_tok * HB;
        const int lo = range_lo(J, c, G), hi = range_lo(J, c + 1, G);
        for (int j0 = lo; j0 < hi; j0 += 64) {
            const int j = j0 + (tid >> 2), q = tid & 3;
            const bool active = j < hi;
            const int jj = active ? j : lo;
            const int t = jj / HB, b = jj - t * HB, ks = b / 16;
            const uint2 xv = __ldg(reinterpret_cast<const uint2*>(P.x + (int64_t)t * P.x_stride + b * 16 + 4 * q));
            float v[4] = {__uint_as_float(xv.x << 16), __uint_as_float(xv.x & 0xffff0000u),
                          __uint_as_float(xv.y << 16), __uint_as_float(xv.y & 0xffff0000u)};
            uint8_t* img = ximg + (int64_t)(t * KSG + ks) * 1024;
            const int sf_off = (int)(xsf - img) + (t * KSG + ks) * 64;
            quant4_put(v, S.xk[t], active, img, 0, sf_off, b % 16);
        }
        fence_proxy_async_global();
        __threadfence();
        named_bar_sync(2, 256);
        if (tid == 0 && hi > lo) red_release_add(phase + PH_X, hi - lo);
    }

    if (warp == 8) {
        // ---- weight producer: the A tiles (codes + pool scales) of every stage in order
        if (lane == 0) {
            const uint64_t pol = l2_evict_first_policy();
            int it = 0;
            bool ok = true;
            for (int k = 0; k < n_units && ok; ++k) {
                int ph, u;
                W.at(k, c, G, ph, u);
                const int KS = ph ? KSD : KSG, UPG = ph ? RB : JB;
                const int g = u / UPG, sub = u - g * UPG;
                const int slot = S.g_sp[g] & 0xffffff, pool = S.g_sp[g] >> 24;
                const CUtensorMap* m = A.map + pool * 6;
                for (int ks = 0; ks < KS; ++ks, ++it) {
                    const int s = it % kNS;
                    if (it >= kNS && !wait_bar(&S.empty[s], ((it / kNS) + 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* st = S.base + s * kStageBytes;
                    mbar_arrive_expect_tx(&S.full[s], 16384 + 2048);
                    if (ph == 0) {
                        tma_load_3d(st, m + M_GATE, ks * 128, sub * 64, slot, &S.full[s], pol);
                        tma_load_3d(st + 8192, m + M_UP, ks * 128, sub * 64, slot, &S.full[s], pol);
                        tma_load_3d(st + kOffASF, m + M_GATE_SF, ks * 16, sub * 64, slot, &S.full[s], pol);
                        tma_load_3d(st + kOffASF + 1024, m + M_UP_SF, ks * 16, sub * 64, slot, &S.full[s], pol);
                    } else {
                        tma_load_3d(st, m + M_DOWN, ks * 128, sub * 128, slot, &S.full[s], pol);
                        tma_load_3d(st + kOffASF, m + M_DOWN_SF, ks * 16, sub * 128, slot, &S.full[s], pol);
                    }
                }
            }
            if (!ok) {
                report_timeout(P);
                // let this CTA's copies in flight land before it leaves (bounded)
                for (int k = std::max(0, it - kNS); k < it; ++k)
                    mbar_wait_bounded(&S.full[k % kNS], (k / kNS) & 1, 1u << 16);
            }
        }
        __syncwarp();
    } else if (warp == 9) {
        // ---- activation-image producer: a stage's B rows once its group's image is ready
        if (lane == 0) {
            int it = 0, ready = -1;
            bool ok = true;
            for (int k = 0; k < n_units && ok; ++k) {
                int ph, u;
                W.at(k, c, G, ph, u);
                const int KS = ph ? KSD : KSG, UPG = ph ? RB : JB;
                const int g = u / UPG;
                const int npad = npad_of(S.g_nt[g]);
                const int key = ph ? g : -2;  // gate_up images: all ready together
                if (key != ready) {
                    const bool r = ph == 0 ? wait_count(phase + PH_X, P.n_tok * HB, abort)
                                           : wait_count(gcnt + 2 * g + 1, S.g_nt[g], abort);
                    if (!r) {
                        ok = false;
                        break;
                    }
                    fence_proxy_async_global();
                    ready = key;
                }
                const int nt = S.g_nt[g], e0 = S.g_e0[g];
                for (int ks = 0; ks < KS; ++ks, ++it) {
                    const int s = it % kNS;
                    if (it >= kNS && !wait_bar(&S.empty[s], ((it / kNS) + 1) & 1, abort)) {
                        ok = false;
                        break;
                    }
                    uint8_t* dst = S.base + s * kStageBytes + kOffB;
                    if (ph) {
                        const uint8_t* src = bimg + ((int64_t)g * KSD + ks) * kFp4ImgStage;
                        mbar_arrive_expect_tx(&S.full[s], npad * 144);
                        bulk_g2s(dst, src, npad * 144, &S.full[s]);
                    } else {
                        // entry i: rows 4 i .. 4 i + 3 (swizzle phase i & 1) and their scales
                        mbar_arrive_expect_tx(&S.full[s], nt * 576);
                        for (int i = 0; i < nt; ++i) {
                            const int t = S.etok[e0 + i];
                            bulk_g2s(dst + i * 512, ximg + ((int64_t)(t * KSG + ks) * 2 + (i & 1)) * 512,
                                     512, &S.full[s]);
                            bulk_g2s(dst + npad * 128 + i * 64, xsf + (int64_t)(t * KSG + ks) * 64, 64,
                                     &S.full[s]);
                        }
                    }
                }
            }
            if (!ok) report_timeout(P);
        }
        __syncwarp();
    } else if (warp == 10) {
        // ---- MMA issuer: 4 MMAs (K 64 each) per stage into the unit's D buffer
        int it = 0;
        bool ok = true;
        for (int k = 0; k < n_units && ok; ++k) {
            int ph, u;
            W.at(k, c, G, ph, u);
            const int KS = ph ? KSD : KSG, UPG = ph ? RB : JB;
            const uint32_t idesc = umma::idesc_mxf4(128, npad_of(S.g_nt[u / UPG]));
            const int db = k % kND;
            if (k >= kND && !wait_bar(&S.d_empty[db], ((k / kND) + 1) & 1, abort)) {
                ok = false;
                break;
            }
            umma::fence_after_sync();
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % kNS;
                if (!wait_bar(&S.sf_full[s], (it / kNS) & 1, abort)) {
                    ok = false;
                    break;
                }
                umma::fence_after_sync();
                if (lane == 0) {
                    const uint32_t sa = smem_u32(S.base + s * kStageBytes);
#pragma unroll
                    for (int i = 0; i < 4; ++i)
                        umma::mma_mxf4(tm + kTmD + db * 32, umma::smem_desc_sw128(sa + 32 * i),
                                       umma::smem_desc_sw128(sa + kOffB + 32 * i), idesc,
                                       tm + kTmSFA + s * 16 + 4 * i, tm + kTmSFB + s * 16 + 4 * i,
                                       (ks == 0 && i == 0) ? 0u : 1u);
                    umma::commit(&S.empty[s]);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) umma::commit(&S.d_full[db]);
            __syncwarp();
        }
        if (!ok) report_timeout(P);
    } else if (warp >= 4) {
        // ---- scale factors: pool scales (A) and activation scales (B) into tensor memory
        const int qd = warp - 4;
        int it = 0;
        bool ok = true;
        for (int k = 0; k < n_units && ok; ++k) {
            int ph, u;
            W.at(k, c, G, ph, u);
            const int KS = ph ? KSD : KSG, UPG = ph ? RB : JB;
            const int npad = npad_of(S.g_nt[u / UPG]);
            for (int ks = 0; ks < KS; ++ks, ++it) {
                const int s = it % kNS;
                if (!wait_bar(&S.full[s], (it / kNS) & 1, abort)) {
                    ok = false;
                    break;
                }
                const uint8_t* st = S.base + s * kStageBytes;
                uint32_t v[16];
#pragma unroll
                for (int m1 = 0; m1 < 4; ++m1) {
                    const uint4 w = *reinterpret_cast<const uint4*>(st + kOffASF + (32 * m1 + lane) * 16);
                    v[m1] = w.x;
                    v[4 + m1] = w.y;
                    v[8 + m1] = w.z;
                    v[12 + m1] = w.w;
                }
                umma::st_x16(tm + ((uint32_t)(qd * 32) << 16) + kTmSFA + s * 16, v);
                uint4 bw = make_uint4(0, 0, 0, 0);
                if (lane < npad) bw = *reinterpret_cast<const uint4*>(st + kOffB + npad * 128 + lane * 16);
                const uint32_t vb[16] = {bw.x, 0, 0, 0, bw.y, 0, 0, 0, bw.z, 0, 0, 0, bw.w, 0, 0, 0};
                umma::st_x16(tm + ((uint32_t)(qd * 32) << 16) + kTmSFB + s * 16, vb);
                umma::wait_st();
                umma::fence_before_sync();
                __syncwarp();
                if (lane == 0) mbar_arrive(&S.sf_full[s]);
            }
        }
        if (!ok) report_timeout(P);
    } else {
        // ---- epilogue warps (TMEM lane quadrants 0-3)
        const int r = tid;  // D row = TMEM lane
        float* ypart = wsp<float>(P, L.ypart);
        float* h32all = wsp<float>(P, L.h32);
        int* hk = wsp<int>(P, L.hk);
        bool ok = true;
        int ke_g = -1, ke[8];
        for (int k = 0; k < n_units && ok; ++k) {
            int ph, u;
            W.at(k, c, G, ph, u);
            const int UPG = ph ? RB : JB;
            const int g = u / UPG, sub = u - g * UPG;
            const int nt = S.g_nt[g], e0 = S.g_e0[g], pool = S.g_sp[g] >> 24;
            const int* d = desc + (int64_t)g * kDescInts;
            // the unit's record fields, loaded while its MMAs run
            int tok[8];
            float wgt[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                tok[i] = i < nt ? __ldcg(d + GD_TOK + i) : 0;
                wgt[i] = i < nt ? __int_as_float(__ldcg(d + GD_W + i)) : 0.f;
            }
            const nvmoe_expert_pool& pl = pool ? P.shared : P.pool;  // (after any refill)
            const int slot = S.g_sp[g] & 0xffffff;
            const float gl = global_of(ph ? pl.down : (r < 64 ? pl.gate : pl.up), slot);
            const int db = k % kND;
            if (!wait_bar(&S.d_full[db], (k / kND) & 1, abort)) {
                ok = false;
                break;
            }
            umma::fence_after_sync();
            uint32_t d0[16], d1[16];
            umma::ld_x16(umma::lane_addr(tm, warp, kTmD + db * 32), d0);
            umma::ld_x16(umma::lane_addr(tm, warp, kTmD + db * 32 + 16), d1);
            umma::wait_ld();
            umma::fence_before_sync();
            __syncwarp();
            if (lane == 0) mbar_arrive(&S.d_empty[db]);
            if (ph == 1 && g != ke_g) {
                // h exponents: written before the group's h-ready count, which this unit's B
                // operand (copied after it) implies
#pragma unroll
                for (int i = 0; i < 8; ++i) ke[i] = i < nt ? __ldcg(hk + g * kGroupMaxTok + i) : 0;
                ke_g = g;
            }
            float v[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {  // column 4 i + t = term t of token i, x 2^(k_i + 2 t)
                float s0 = 0.f, s1 = 0.f;
#pragma unroll
                for (int t = kFp4Terms - 1; t >= 0; --t) {
                    s0 = fmaf(__uint_as_float(d0[kFp4Terms * i + t]), fp4_exp2(-2 * t), s0);
                    s1 = fmaf(__uint_as_float(d1[kFp4Terms * i + t]), fp4_exp2(-2 * t), s1);
                }
                const int k0 = ph ? ke[i] : S.xk[tok[i]], k1 = ph ? ke[4 + i] : S.xk[tok[4 + i]];
                v[i] = s0 * fp4_exp2(-k0);
                v[4 + i] = s1 * fp4_exp2(-k1);
            }
            if (ph == 1) {
                // down: the weighted rows of the group's entries for H rows [128 sub, +128)
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (i >= nt) break;
                    const float w = wgt[i] * gl * (pool ? S.sg[tok[i]] : 1.0f);
                    ypart[(int64_t)(e0 + i) * H + sub * 128 + r] = v[i] * w;
                }
                continue;
            }
            // gate_up: gate rows 0-63, up rows 64-127 of j = 64 sub + (r % 64) -> h (fp32)
            if (r >= 64) {
#pragma unroll
                for (int i = 0; i < 8; ++i) S.xbuf[(r - 64) * 8 + i] = v[i] * gl;
            }
            named_bar_sync(1, 128);
            float* h32 = h32all + (int64_t)g * kGroupMaxTok * I;
            if (r < 64) {
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    if (i >= nt) break;
                    h32[(int64_t)i * I + sub * 64 + r] = silu(v[i] * gl) * S.xbuf[r * 8 + i];
                }
            }
            __threadfence();
            named_bar_sync(1, 128);
            // h rows: the group's last j-block to be stored (it finds the count at JB - 1; the
            // others are all in memory) builds every row.  Thread tid owns the 4 values
            // [4 tid + 512 m, +4) of each row (m < I / 512): the 4 lanes of a 16-block, as
            // quant4_put wants them.  Pass 1: the row maxima (warp, then block); pass 2: each
            // 16-block as 4 NVFP4 terms in the group's down image, the exponents in hk.
            if (tid == 0) {
                const int old = atomicAdd(gcnt + 2 * g, 1);
                __threadfence();
                S.misc[0] = old == JB - 1 ? 1 : 0;
            }
            named_bar_sync(1, 128);
            if (S.misc[0]) {
                const int MC = (I + 511) / 512, npad = npad_of(nt);  // I a multiple of 256
                float* rmax = S.xbuf;                                 // [4 warps][8 rows]
                float4 keep[8];  // chunk 0 of every row (all loads of a chunk in flight at once)
                float am[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) am[i] = 0.f;
                for (int m = 0; m < MC; ++m) {
                    const bool valid = 4 * tid + 512 * m < I;
                    float4 f[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        f[i] = (i < nt && valid) ? __ldcg(reinterpret_cast<const float4*>(h32 + (int64_t)i * I + 512 * m) + tid)
                                                 : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        am[i] = fmaxf(am[i], fmaxf(fmaxf(fabsf(f[i].x), fabsf(f[i].y)), fmaxf(fabsf(f[i].z), fabsf(f[i].w))));
                        if (m == 0) keep[i] = f[i];
                    }
                }
#pragma unroll
                for (int o = 16; o > 0; o >>= 1)
#pragma unroll
                    for (int i = 0; i < 8; ++i) am[i] = fmaxf(am[i], __shfl_xor_sync(0xffffffffu, am[i], o));
                if (lane == 0)
#pragma unroll
                    for (int i = 0; i < 8; ++i) rmax[warp * 8 + i] = am[i];
                named_bar_sync(1, 128);
                int kh[8];
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    kh[i] = fp4_row_exp(fmaxf(fmaxf(rmax[i], rmax[8 + i]), fmaxf(rmax[16 + i], rmax[24 + i])));
                    if (tid == 0 && i < nt) hk[g * kGroupMaxTok + i] = kh[i];
                }
                for (int m = 0; m < MC; ++m) {
                    const bool valid = 4 * tid + 512 * m < I;
                    float4 f[8];
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        f[i] = m == 0 ? keep[i]
                             : ((i < nt && valid) ? __ldcg(reinterpret_cast<const float4*>(h32 + (int64_t)i * I + 512 * m) + tid)
                                                  : make_float4(0.f, 0.f, 0.f, 0.f));
                    const int blk = valid ? (tid >> 2) + 32 * m : 0;
                    uint8_t* img = bimg + ((int64_t)g * KSD + blk / 16) * kFp4ImgStage;
#pragma unroll
                    for (int i = 0; i < 8; ++i) {
                        if (i >= nt) break;
                        float v4[4] = {f[i].x, f[i].y, f[i].z, f[i].w};
                        quant4_put(v4, kh[i], valid, img, npad, i, blk % 16);
                    }
                }
                fence_proxy_async_global();
                __threadfence();
                named_bar_sync(1, 128);
                if (tid == 0) red_release_add(gcnt + 2 * g + 1, nt);
            }
        }
        // every entry row is stored: this CTA's slice of y = sum over j = 0..k (shared last)
        if (ok && NG) {
            named_bar_sync(1, 128);
            if (tid == 0) {
                __threadfence();
                red_release_add(phase + PH_DN, 1);
                ok = wait_count(phase + PH_DN, G, abort);
                __threadfence();
            }
            named_bar_sync(1, 128);
        }
        if (ok && NG) {
            const int n_out = P.n_tok * H;
            const int lo = range_lo(n_out, c, G), hi = range_lo(n_out, c + 1, G);
            for (int o = lo + tid; o < hi; o += 128) {
                const int t = o / H, col = o - t * H;
                float vals[kMaxK1];
#pragma unroll
                for (int j = 0; j < kMaxK1; ++j) {
                    const int e = j < K1 ? S.ent[t * K1 + j] : -1;
                    vals[j] = e >= 0 ? __ldcg(ypart + (int64_t)e * H + col) : 0.f;
                }
                float sum = 0.f;
#pragma unroll
                for (int j = 0; j < kMaxK1; ++j) sum += vals[j];
                P.y[(int64_t)t * P.y_stride + col] = f32_to_bf16_bits(sum);
            }
        }
        if (!ok) report_timeout(P);
    }

    umma::fence_before_sync();
    __syncthreads();
    if (warp == 10) {
        umma::fence_after_sync();
        umma::tmem_dealloc(tm, kTmCols);
    }
}

// ------------------------------------------------------------------ host: tensor maps
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encoder() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

using MapKey = std::tuple<uintptr_t, uint64_t, uint64_t, uint64_t, uint64_t, uint64_t, uint32_t,
                          uint32_t>;
std::mutex g_map_mu;
std::map<MapKey, CUtensorMap> g_maps;

// 3-D map over a bank: (bytes of a row, rows, slots), box (box_bytes, box_rows, 1), uint8.
bool bank_map(CUtensorMap* out, const void* base, uint64_t row_bytes, uint64_t rows,
              uint64_t slots, uint64_t row_stride, uint64_t slot_stride, uint32_t box_bytes,
              uint32_t box_rows, bool swizzle) {
    if (!base || (reinterpret_cast<uintptr_t>(base) & 15) || (row_stride & 15) ||
        row_stride < row_bytes || rows < box_rows || row_bytes < box_bytes)
        return false;
    if (slots <= 1) {
        slots = 1;
        slot_stride = rows * row_stride;
    }
    if ((slot_stride & 15) || slot_stride < rows * row_stride) return false;
    const MapKey key{reinterpret_cast<uintptr_t>(base), row_bytes, rows, slots, row_stride,
                     slot_stride, box_bytes, box_rows | (swizzle ? 0x80000000u : 0u)};
    std::lock_guard<std::mutex> lk(g_map_mu);
    auto itm = g_maps.find(key);
    if (itm != g_maps.end()) {
        *out = itm->second;
        return true;
    }
    EncodeTiledFn enc = encoder();
    if (!enc) return false;
    const cuuint64_t dims[3] = {row_bytes, rows, slots};
    const cuuint64_t strides[2] = {row_stride, slot_stride};
    const cuuint32_t box[3] = {box_bytes, box_rows, 1};
    const cuuint32_t est[3] = {1, 1, 1};
    CUtensorMap m;
    std::memset(&m, 0, sizeof(m));
    const CUresult r = enc(&m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, const_cast<void*>(base), dims,
                           strides, box, est, CU_TENSOR_MAP_INTERLEAVE_NONE,
                           swizzle ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return false;
    if (g_maps.size() > 4096) g_maps.clear();
    g_maps.emplace(key, m);
    *out = m;
    return true;
}

}  // namespace

bool fp4_pool_maps(const nvmoe_expert_pool& p, CUtensorMap* m) {
    const int H = p.hidden, I = p.inter;
    const uint64_t S = (uint64_t)p.n_slots;
    return bank_map(m + M_GATE, p.gate.data, H / 2, I, S, p.gate.row_stride, p.gate.slot_stride,
                    128, 64, true) &&
           bank_map(m + M_GATE_SF, p.gate.scale, H / 16, I, S, p.gate.scale_row_stride,
                    p.gate.scale_slot_stride, 16, 64, false) &&
           bank_map(m + M_UP, p.up.data, H / 2, I, S, p.up.row_stride, p.up.slot_stride, 128, 64,
                    true) &&
           bank_map(m + M_UP_SF, p.up.scale, H / 16, I, S, p.up.scale_row_stride,
                    p.up.scale_slot_stride, 16, 64, false) &&
           bank_map(m + M_DOWN, p.down.data, I / 2, H, S, p.down.row_stride,
                    p.down.slot_stride, 128, 128, true) &&
           bank_map(m + M_DOWN_SF, p.down.scale, I / 16, H, S, p.down.scale_row_stride,
                    p.down.scale_slot_stride, 16, 128, false);
}


// Whether a call runs on the FP4 tensor-core kernel (decided in ffn_setup, so the kernels
// before it know whether to write the f16 token copy): NVFP4 pools whose shapes it covers, when
// the call asks for it (nvmoe_ffn_args.kernel == NVMOE_KERNEL_FP4).  By default the mma.sync kernel runs:
// measured at batch 8 on the Qwen3.8-shaped layer it is faster (the FP4 kernel's per-unit
// epilogue handoffs between CTAs cost more than its dequantisation-free stream saves).
bool ffn_fp4_eligible(const FfnParams& P) {
    if (P.pool.quant != NVMOE_Q_NVFP4 || P.L.jb == 0) return false;
    if (P.n_tok > kMaxTok || P.L.g_max > kMaxGroups) return false;
    if (P.n_tok * (P.top_k + 1) > kMaxEntOf || P.top_k + 1 > kMaxK1) return false;

    // 32-bit range arithmetic: (stages or outputs) x (CTAs + 1) < 2^32
    const uint64_t units = (uint64_t)P.L.g_max * std::max(P.L.jb * P.L.ks_gu, P.L.rb);
    if (units * (kFp4MaxCtas + 1) >= (1ull << 32) ||
        (uint64_t)P.n_tok * P.pool.hidden * (kFp4MaxCtas + 1) >= (1ull << 32))
        return false;
    if (P.x_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(P.x) & 15)) return false;
    if (P.kernel != NVMOE_KERNEL_FP4) return false;
    CUtensorMap m[6];
    if (!fp4_pool_maps(P.pool, m)) return false;
    if (P.has_shared && !fp4_pool_maps(P.shared, m)) return false;
    int dev = 0, sms = 0;
    if (cudaGetDevice(&dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
        return false;
    // a group's j-blocks sit on distinct CTAs (its h rows wait for all of them)
    return sms > 0 && sms <= kFp4MaxCtas && sms >= P.L.jb;
}

int ffn_fp4_launch(const FfnParams& P, cudaStream_t st) {
    Fp4Params A;
    std::memset(&A, 0, sizeof(A));
    A.P = P;
    if (!fp4_pool_maps(P.pool, A.map)) return NVMOE_ERR_UNSUPPORTED;
    if (!fp4_pool_maps(P.has_shared ? P.shared : P.pool, A.map + 6)) return NVMOE_ERR_UNSUPPORTED;
    int dev = 0, sms = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    NVMOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_fp4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        kSmemTotal));
    // one CTA per SM (shared memory) and no more CTAs than SMs: every CTA is resident, so the
    // waits on other CTAs' images and partial tiles end
    const cudaError_t e = launch_pdl(ffn_fp4_kernel, dim3(std::min(sms, kFp4MaxCtas)),
                                     dim3(kThreads), (size_t)kSmemTotal, st, true, A);
    return cuda_status("ffn_fp4 launch", e);
}

}  // namespace nvmoe
