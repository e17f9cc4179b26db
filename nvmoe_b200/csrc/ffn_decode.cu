// R7 / R9 — routed-expert FFN over the slot pool for decode-sized batches.
//
// Reference call: _expert_gemm(cache, hidden, topk_weights, slot_ids, views, n, alphas,
// is_prefill) (nvme-moe-bench/nvme_offload_cache.py:1989-1998, 2165-2174) and ggml mul_mat_id
// over the reduced [.., .., cache_size] expert tensors (scripts/test_mul_mat_id_shrink.cpp:29-69):
//   y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] ),  s = slot_ids[t, j]
// plus the always-on shared expert (nvme_offload_cache.py:2115-2123).
//
// Kernels (chained with programmatic dependent launch):
//   prep    — x -> f16, shared-expert gate, grouping of the (token, k) entries by slot into
//             token groups of <= 8 entries (ffn_common.cuh); the fused decode front kernel does
//             the same work in the engine path
//   gate_up — persistent, 1 CTA / SM: a producer warp streams work items (token group, 16 rows of
//             gate + the same rows of up) with 1-D bulk copies (TMA) into a ring of shared-memory
//             stages; 8 consumer warps split K, dequantise A fragments in registers from the
//             staged bytes, run m16n8k16 f16 MMAs (fp32 accumulate), reduce across warps and
//             write h = silu(g) * u (f16) per entry
//   down    — one CTA per 16 output rows: the producer streams every token group's 16 down rows
//             (issued before the grid-dependency wait: weights do not depend on gate_up) and its
//             h rows; each consumer warp owns whole groups (full K), writes w * down(h) per entry
//             into shared memory, and the CTA finally sums the entries of each token in the
//             fixed order j = 0..k-1, shared, and stores bf16 y.  No atomics, deterministic.
// Only the slots that occur in slot_ids are read; every weight byte is read once per call.
#include "common.cuh"
#include "dequant_frag.cuh"
#include "ffn_common.cuh"

#include <algorithm>

namespace nvmoe {
namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kTmaThreads = kConsumers + 32;  // + one producer warp
constexpr int kSmemCap = 227 * 1024 - 1024;   // dynamic share; static use stays below 1 KB
constexpr int kStageHdr = 128;  // per stage: group descriptor + scalars fetched by the producer
constexpr int kHdrExt = 10;     // header floats after the descriptor (see load_desc_ext)

// ------------------------------------------------------------------ 1. prep
__global__ void __launch_bounds__(kPrepThreads) ffn_prep_kernel(FfnParams P) {
    extern __shared__ __align__(16) int prep_smem[];
    grid_dep_wait();
    grid_dep_launch();
    if ((int)blockIdx.x < (int)gridDim.x - 1) {
        ffn_convert_tokens(P, blockIdx.x, gridDim.x - 1);
    } else {
        ffn_group_block(P, prep_smem);
    }
}

__device__ __forceinline__ void report_timeout(const FfnParams& P) {
    atomicExch(wsp<int>(P, P.L.hdr) + HDR_STATUS, NVMOE_ERR_TIMEOUT);
    if (P.status) atomicExch(P.status, NVMOE_ERR_TIMEOUT);
}

// Copies `rows` rows of `row_bytes` from a bank (row stride `stride`) into contiguous smem.
__device__ __forceinline__ void bulk_rows(uint8_t* dst, const uint8_t* src, int rows,
                                          int row_bytes, int64_t stride, uint64_t* bar) {
    if (stride == row_bytes) {
        bulk_g2s(dst, src, (uint32_t)(rows * row_bytes), bar);
    } else {
        for (int r = 0; r < rows; ++r)
            bulk_g2s(dst + r * row_bytes, src + r * stride, (uint32_t)row_bytes, bar);
    }
}

// Loads the descriptor of group `grp` (16 ints) with L2 reads.
__device__ __forceinline__ void load_desc(const FfnParams& P, int grp, int (&d)[kDescInts]) {
    const int4* src = reinterpret_cast<const int4*>(wsp<int>(P, P.L.grp_desc) +
                                                    (int64_t)grp * kDescInts);
#pragma unroll
    for (int i = 0; i < kDescInts / 4; ++i) {
        const int4 v = __ldcg(src + i);
        d[4 * i] = v.x, d[4 * i + 1] = v.y, d[4 * i + 2] = v.z, d[4 * i + 3] = v.w;
    }
}

__device__ __forceinline__ float global_of(const nvmoe_matrix_bank& b, int slot) {
    return b.global_scale ? __ldcg(b.global_scale + (int64_t)slot * b.global_stride) : 1.0f;
}

// Scalars an item needs in its epilogue, fetched by the producer lanes in parallel (off the
// consumers' critical path) and shipped in the stage header after the descriptor:
//   gate_up: ext[0] = gate global, ext[1] = up global
//   down   : ext[0] = down global, ext[2 + n] = combine weight of entry n (times the shared
//            expert's sigmoid gate for the shared pool)
template <bool kDown>
__device__ __forceinline__ void load_desc_ext(const FfnParams& P, int grp, int (&d)[kDescInts],
                                              float (&ext)[kHdrExt]) {
    load_desc(P, grp, d);
    const nvmoe_expert_pool& pool = d[GD_POOL] ? P.shared : P.pool;
#pragma unroll
    for (int i = 0; i < kHdrExt; ++i) ext[i] = 0.f;
    if (!kDown) {
        ext[0] = global_of(pool.gate, d[GD_SLOT]);
        ext[1] = global_of(pool.up, d[GD_SLOT]);
    } else {
        ext[0] = global_of(pool.down, d[GD_SLOT]);
        const float* ent_w = wsp<float>(P, P.L.ent_w);
        const float* sgv = (d[GD_POOL] && P.shared_gate) ? wsp<float>(P, P.L.sg) : nullptr;
#pragma unroll
        for (int n = 0; n < kGroupMaxTok; ++n) {
            if (n < d[GD_NT]) {
                float w = __ldcg(ent_w + d[GD_E0] + n);
                if (sgv) w *= __ldcg(sgv + d[GD_TOK + n]);
                ext[2 + n] = w;
            }
        }
    }
}

// ------------------------------------------------------------------ 2. gate_up + SwiGLU
// Stage layout: [hdr 64 B] gate codes [16][H/2] | up codes | gate scales [16][H/16] |
// up scales | x [8][H] f16.
template <typename Fmt>
__global__ void __launch_bounds__(kTmaThreads, 1) ffn_gate_up_tma(FfnParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int NST = P.nst_gu;
    const int stage_bytes = P.stage_gu;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NST * stage_bytes);
    uint64_t* empty = full + NST;
    float* red = reinterpret_cast<float*>(empty + NST);  // [8 warps][32 lanes][8]
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        mbar_init_fence();
    }
    __syncthreads();
    grid_dep_wait();
    grid_dep_launch();

    const int tiles = I / 16;
    const int n_groups = __ldcg(wsp<int>(P, P.L.hdr) + HDR_N_GROUPS);
    const int n_items = n_groups * tiles;
    const int cb = Fmt::code_bytes(H), sb = Fmt::scale_bytes(H);
    const int off_codes = kStageHdr, off_ucodes = kStageHdr + 16 * cb;
    const int off_gsc = kStageHdr + 32 * cb, off_usc = off_gsc + 16 * sb;
    const int off_x = off_usc + 16 * sb;
    const __half* x16 = wsp<__half>(P, P.L.x16);

    if (warp == kConsumerWarps) {
        // ---------------- producer: descriptors of 32 items at a time, one per lane
        int it = 0;
        bool ok = true;
        for (int base = blockIdx.x; base < n_items && ok; base += 32 * gridDim.x) {
            const int my_item = base + lane * gridDim.x;
            int d[kDescInts];
            float ext[kHdrExt];
            if (my_item < n_items) load_desc_ext<false>(P, my_item / tiles, d, ext);
            const int n_here = min(32, (n_items - base + (int)gridDim.x - 1) / (int)gridDim.x);
            for (int i = 0; i < n_here; ++i, ++it) {
                int dd[kDescInts];
                float ee[kHdrExt];
#pragma unroll
                for (int k = 0; k < kDescInts; ++k) dd[k] = __shfl_sync(0xffffffffu, d[k], i);
#pragma unroll
                for (int k = 0; k < kHdrExt; ++k) ee[k] = __shfl_sync(0xffffffffu, ext[k], i);
                if (lane == 0) {
                    const int item = base + i * gridDim.x;
                    const int st = it % NST;
                    const uint32_t ph = (it / NST) & 1;
                    if (!mbar_wait_bounded(&empty[st], ph ^ 1)) {
                        report_timeout(P);
                        ok = false;
                    } else {
                        const int rt = item % tiles;
                        const nvmoe_expert_pool& pool = dd[GD_POOL] ? P.shared : P.pool;
                        const int slot = dd[GD_SLOT], nt = dd[GD_NT];
                        uint8_t* stg = smem + (size_t)st * stage_bytes;
                        int* hdr = reinterpret_cast<int*>(stg);
#pragma unroll
                        for (int k = 0; k < kDescInts; ++k) hdr[k] = dd[k];
#pragma unroll
                        for (int k = 0; k < kHdrExt; ++k)
                            reinterpret_cast<float*>(hdr + kDescInts)[k] = ee[k];
                        mbar_arrive_expect_tx(&full[st], (uint32_t)(32 * cb + 32 * sb + nt * H * 2));
                        const int64_t r0 = (int64_t)rt * 16;
                        bulk_rows(stg + off_codes,
                                  (const uint8_t*)pool.gate.data + slot * pool.gate.slot_stride +
                                      r0 * pool.gate.row_stride,
                                  16, cb, pool.gate.row_stride, &full[st]);
                        bulk_rows(stg + off_ucodes,
                                  (const uint8_t*)pool.up.data + slot * pool.up.slot_stride +
                                      r0 * pool.up.row_stride,
                                  16, cb, pool.up.row_stride, &full[st]);
                        bulk_rows(stg + off_gsc,
                                  (const uint8_t*)pool.gate.scale + slot * pool.gate.scale_slot_stride +
                                      r0 * pool.gate.scale_row_stride,
                                  16, sb, pool.gate.scale_row_stride, &full[st]);
                        bulk_rows(stg + off_usc,
                                  (const uint8_t*)pool.up.scale + slot * pool.up.scale_slot_stride +
                                      r0 * pool.up.scale_row_stride,
                                  16, sb, pool.up.scale_row_stride, &full[st]);
                        for (int n = 0; n < nt; ++n)
                            bulk_g2s(stg + off_x + n * H * 2, x16 + (int64_t)dd[GD_TOK + n] * H,
                                     (uint32_t)(H * 2), &full[st]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        return;
    }

    // ---------------- consumers
    const int g = lane >> 2, q = lane & 3;
    const int KW = H / kConsumerWarps;
    __half* h16 = wsp<__half>(P, P.L.h16);
    int it = 0;
    for (int item = blockIdx.x; item < n_items; item += gridDim.x, ++it) {
        const int st = it % NST;
        const uint32_t ph = (it / NST) & 1;
        if (!mbar_wait_bounded(&full[st], ph)) {
            report_timeout(P);
            break;
        }
        const int rt = item % tiles;
        const uint8_t* stg = smem + (size_t)st * stage_bytes;
        const int* hdr = reinterpret_cast<const int*>(stg);
        const int e0 = hdr[GD_E0], nt = hdr[GD_NT];
        // the stage is released before the epilogue: keep its scalars in registers
        const float gglob = reinterpret_cast<const float*>(hdr + kDescInts)[0];
        const float uglob = reinterpret_cast<const float*>(hdr + kDescInts)[1];
        const __half* xs = reinterpret_cast<const __half*>(stg + off_x) + g * H;
        const bool has_tok = g < nt;
        float accg[4] = {0.f, 0.f, 0.f, 0.f}, accu[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k0 = warp * KW; k0 < (warp + 1) * KW; k0 += Fmt::kWarpTileK) {
            typename Fmt::Row ga, gb, ua, ub;
            Fmt::load_smem(ga, stg + off_codes + g * cb, stg + off_gsc + g * sb, k0, q);
            Fmt::load_smem(gb, stg + off_codes + (g + 8) * cb, stg + off_gsc + (g + 8) * sb, k0, q);
            Fmt::load_smem(ua, stg + off_ucodes + g * cb, stg + off_usc + g * sb, k0, q);
            Fmt::load_smem(ub, stg + off_ucodes + (g + 8) * cb, stg + off_usc + (g + 8) * sb, k0, q);
#pragma unroll
            for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
                const uint4 xb = has_tok
                                     ? *reinterpret_cast<const uint4*>(xs + k0 + Fmt::kofs(q, s2))
                                     : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int ss = 0; ss < 2; ++ss) {
                    uint32_t ag[4], au[4];
                    Fmt::deq(ga, s2 + ss, ag[0], ag[2]);
                    Fmt::deq(gb, s2 + ss, ag[1], ag[3]);
                    Fmt::deq(ua, s2 + ss, au[0], au[2]);
                    Fmt::deq(ub, s2 + ss, au[1], au[3]);
                    const uint32_t b0 = ss ? xb.z : xb.x, b1 = ss ? xb.w : xb.y;
                    mma_f16_16816(accg, ag, b0, b1);
                    mma_f16_16816(accu, au, b0, b1);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);  // the stage can be refilled
        float* rw = red + (warp * 32 + lane) * 8;
#pragma unroll
        for (int v = 0; v < 4; ++v) rw[v] = accg[v], rw[4 + v] = accu[v];
        named_bar_sync(1, kConsumers);
        if (tid < 128) {
            const int l = tid >> 2, v = tid & 3;
            float sg_ = 0.f, su_ = 0.f;
#pragma unroll
            for (int w = 0; w < kConsumerWarps; ++w) {
                sg_ += red[(w * 32 + l) * 8 + v];
                su_ += red[(w * 32 + l) * 8 + 4 + v];
            }
            const int row = (l >> 2) + ((v >> 1) << 3);
            const int n = 2 * (l & 3) + (v & 1);
            if (n < nt) {
                const float hv = silu(sg_ * gglob) * (su_ * uglob);
                h16[(int64_t)(e0 + n) * I + rt * 16 + row] = __float2half_rn(hv);
            }
        }
        named_bar_sync(1, kConsumers);
    }
}

// ------------------------------------------------------------------ 3. down + combine
// Stage layout: [hdr 64 B] codes [16][I/2] | scales [16][I/16] | h [8][I] f16.
template <typename Fmt>
__global__ void __launch_bounds__(kTmaThreads, 1) ffn_down_tma(FfnParams P) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int NST = P.nst_dn;
    const int stage_bytes = P.stage_dn;
    const int rb = blockIdx.x;  // rows [16 rb, 16 rb + 16)
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + (size_t)NST * stage_bytes);
    uint64_t* empty = full + NST;
    float* yps = reinterpret_cast<float*>(empty + NST);  // [n_ent][16] when in shared memory
    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);  // one consumer warp per stage use
        }
        mbar_init_fence();
    }
    __syncthreads();
    // the group tables come from prep / the front kernel, which completed before the gate_up
    // grid could pass its own dependency wait; h comes from gate_up (read after grid_dep_wait)
    const int n_groups = __ldcg(wsp<int>(P, P.L.hdr) + HDR_N_GROUPS);
    const int cb = Fmt::code_bytes(I), sb = Fmt::scale_bytes(I);
    const int off_codes = kStageHdr, off_sc = kStageHdr + 16 * cb, off_h = off_sc + 16 * sb;
    const __half* h16 = wsp<__half>(P, P.L.h16);

    if (warp == kConsumerWarps) {
        // ---------------- producer
        const int n_first = min(n_groups, NST);
        int d[kDescInts];
        float ext[kHdrExt];
        bool ok = true;
        for (int base = 0; base < n_groups && ok; base += 32) {
            if (base + lane < n_groups) load_desc_ext<true>(P, base + lane, d, ext);
            const int n_here = min(32, n_groups - base);
            for (int i = 0; i < n_here; ++i) {
                const int g = base + i;
                int dd[kDescInts];
                float ee[kHdrExt];
#pragma unroll
                for (int k = 0; k < kDescInts; ++k) dd[k] = __shfl_sync(0xffffffffu, d[k], i);
#pragma unroll
                for (int k = 0; k < kHdrExt; ++k) ee[k] = __shfl_sync(0xffffffffu, ext[k], i);
                if (lane == 0) {
                    const int st = g % NST;
                    const uint32_t ph = (g / NST) & 1;
                    if (!mbar_wait_bounded(&empty[st], ph ^ 1)) {
                        report_timeout(P);
                        ok = false;
                    } else {
                        const nvmoe_expert_pool& pool = dd[GD_POOL] ? P.shared : P.pool;
                        const int slot = dd[GD_SLOT], nt = dd[GD_NT];
                        uint8_t* stg = smem + (size_t)st * stage_bytes;
                        int* hdr = reinterpret_cast<int*>(stg);
#pragma unroll
                        for (int k = 0; k < kDescInts; ++k) hdr[k] = dd[k];
#pragma unroll
                        for (int k = 0; k < kHdrExt; ++k)
                            reinterpret_cast<float*>(hdr + kDescInts)[k] = ee[k];
                        mbar_arrive_expect_tx(&full[st], (uint32_t)(16 * (cb + sb) + nt * I * 2));
                        const int64_t r0 = (int64_t)rb * 16;
                        bulk_rows(stg + off_codes,
                                  (const uint8_t*)pool.down.data + slot * pool.down.slot_stride +
                                      r0 * pool.down.row_stride,
                                  16, cb, pool.down.row_stride, &full[st]);
                        bulk_rows(stg + off_sc,
                                  (const uint8_t*)pool.down.scale + slot * pool.down.scale_slot_stride +
                                      r0 * pool.down.scale_row_stride,
                                  16, sb, pool.down.scale_row_stride, &full[st]);
                        if (g >= n_first)
                            bulk_g2s(stg + off_h, h16 + (int64_t)dd[GD_E0] * I,
                                     (uint32_t)(nt * I * 2), &full[st]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
                if (g == n_first - 1) {
                    // every first-round stage has its weights in flight; now wait for gate_up
                    grid_dep_wait();
                    if (lane == 0)
                        for (int gg = 0; gg < n_first; ++gg) {
                            const int* hdr =
                                reinterpret_cast<const int*>(smem + (size_t)gg * stage_bytes);
                            bulk_g2s(smem + (size_t)gg * stage_bytes + off_h,
                                     h16 + (int64_t)hdr[GD_E0] * I, (uint32_t)(hdr[GD_NT] * I * 2),
                                     &full[gg]);
                        }
                }
            }
        }
        if (n_groups == 0) grid_dep_wait();
        return;
    }

    // ---------------- consumers: warp w owns groups w, w + 8, ...
    grid_dep_wait();
    if (n_groups == 0) {  // no valid entry and no shared expert (or an upstream error): y = 0
        for (int idx = tid; idx < P.n_tok * 16; idx += kConsumers)
            P.y[(int64_t)(idx >> 4) * P.y_stride + rb * 16 + (idx & 15)] = 0;
        return;
    }
    const int g = lane >> 2, q = lane & 3;
    float* ypart = P.ypart_smem ? yps : wsp<float>(P, P.L.ypart);
    const int ypstride = P.ypart_smem ? 16 : H;  // floats between entries
    const int ypcol = P.ypart_smem ? 0 : rb * 16;
    const int* ent_of = wsp<int>(P, P.L.ent_of);
    for (int grp = warp; grp < n_groups; grp += kConsumerWarps) {
        const int st = grp % NST;
        const uint32_t ph = (grp / NST) & 1;
        if (!mbar_wait_bounded(&full[st], ph)) {
            report_timeout(P);
            break;
        }
        const uint8_t* stg = smem + (size_t)st * stage_bytes;
        const int* hdr = reinterpret_cast<const int*>(stg);
        const int e0 = hdr[GD_E0], nt = hdr[GD_NT];
        // the stage is released before the epilogue: keep its scalars in registers
        const float* ext_s = reinterpret_cast<const float*>(hdr + kDescInts);
        const float dglob = ext_s[0];
        const float w_lo = ext_s[2 + 2 * q], w_hi = ext_s[3 + 2 * q];  // tokens 2q, 2q+1
        const __half* hs = reinterpret_cast<const __half*>(stg + off_h) + g * I;
        const bool has_tok = g < nt;
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int k0 = 0; k0 < I; k0 += Fmt::kWarpTileK) {
            typename Fmt::Row ra, rbw;
            Fmt::load_smem(ra, stg + off_codes + g * cb, stg + off_sc + g * sb, k0, q);
            Fmt::load_smem(rbw, stg + off_codes + (g + 8) * cb, stg + off_sc + (g + 8) * sb, k0, q);
#pragma unroll
            for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
                const uint4 hb = has_tok
                                     ? *reinterpret_cast<const uint4*>(hs + k0 + Fmt::kofs(q, s2))
                                     : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int ss = 0; ss < 2; ++ss) {
                    uint32_t af[4];
                    Fmt::deq(ra, s2 + ss, af[0], af[2]);
                    Fmt::deq(rbw, s2 + ss, af[1], af[3]);
                    mma_f16_16816(acc, af, ss ? hb.z : hb.x, ss ? hb.w : hb.y);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st]);
        // C fragment: rows g, g+8; tokens 2q, 2q+1 of the group
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const int row = g + ((v >> 1) << 3);
            const int n = 2 * q + (v & 1);
            if (n < nt) {
                const int e = e0 + n;
                ypart[(int64_t)e * ypstride + ypcol + row] = acc[v] * dglob * ((v & 1) ? w_hi : w_lo);
            }
        }
    }
    named_bar_sync(1, kConsumers);
    // y rows of this CTA: entries of each token summed in the order j = 0..k-1, shared
    const int K1 = P.top_k + 1;
    for (int idx = tid; idx < P.n_tok * 16; idx += kConsumers) {
        const int t = idx >> 4, r = idx & 15;
        float sum = 0.f;
        for (int j = 0; j < K1; ++j) {
            const int e = ent_of[t * K1 + j];
            if (e >= 0) sum += ypart[(int64_t)e * ypstride + ypcol + r];
        }
        P.y[(int64_t)t * P.y_stride + rb * 16 + r] = f32_to_bf16_bits(sum);
    }
}

bool pool_ok(const nvmoe_expert_pool& p) {
    return p.gate.data && p.up.data && p.down.data && p.hidden > 0 && p.inter > 0 &&
           p.n_slots > 0;
}

// Rows are staged with 1-D bulk copies (TMA), which need 16-byte aligned addresses and sizes;
// reject any bank whose base or strides would break that alignment.
bool bank_aligned(const nvmoe_matrix_bank& b, bool nvfp4) {
    const uintptr_t d = reinterpret_cast<uintptr_t>(b.data);
    if ((d & 15) || (b.slot_stride & 15) || (b.row_stride & 15)) return false;
    if (nvfp4) {
        const uintptr_t s = reinterpret_cast<uintptr_t>(b.scale);
        if (!b.scale || (s & 15) || (b.scale_slot_stride & 15) || (b.scale_row_stride & 15))
            return false;
    }
    return true;
}

bool pool_aligned(const nvmoe_expert_pool& p) {
    const bool nv = p.quant == NVMOE_Q_NVFP4;
    return bank_aligned(p.gate, nv) && bank_aligned(p.up, nv) && bank_aligned(p.down, nv);
}

template <typename Fmt>
int launch_fmt(FfnParams& P, cudaStream_t st) {
    const int H = P.pool.hidden, I = P.pool.inter;
    const int red_gu = kConsumerWarps * 32 * 8 * 4;
    const int sgu = kStageHdr + 32 * Fmt::code_bytes(H) + 32 * Fmt::scale_bytes(H) +
                    kGroupMaxTok * H * 2;
    const int nst_gu = std::min(4, (kSmemCap - red_gu - 1024) / sgu);
    const int sdn = kStageHdr + 16 * (Fmt::code_bytes(I) + Fmt::scale_bytes(I)) +
                    kGroupMaxTok * I * 2;
    const size_t yp_bytes = (size_t)P.L.n_ent_max * 16 * 4;
    P.ypart_smem = (yp_bytes + 4 * (size_t)sdn + 1024 <= (size_t)kSmemCap) ? 1 : 0;
    const size_t yp_used = P.ypart_smem ? yp_bytes : 0;
    const int nst_dn = (int)std::min<size_t>(16, (kSmemCap - yp_used - 1024) / sdn);
    if (nst_gu < 1 || nst_dn < 2) return NVMOE_ERR_UNSUPPORTED;
    P.nst_gu = nst_gu;
    P.stage_gu = sgu;
    P.nst_dn = nst_dn;
    P.stage_dn = sdn;
    const size_t smem_gu = (size_t)nst_gu * sgu + 16 * nst_gu + red_gu;
    const size_t smem_dn = (size_t)nst_dn * sdn + 16 * nst_dn + yp_used;
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_gate_up_tma<Fmt>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_gu));
    NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_down_tma<Fmt>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dn));
    cudaError_t e =
        launch_pdl(ffn_gate_up_tma<Fmt>, dim3(kNumSMs), dim3(kTmaThreads), smem_gu, st, true, P);
    if (e != cudaSuccess) return cuda_status("ffn_gate_up launch", e);
    e = launch_pdl(ffn_down_tma<Fmt>, dim3(H / 16), dim3(kTmaThreads), smem_dn, st, true, P);
    return cuda_status("ffn_down launch", e);
}

}  // namespace

int ffn_setup(const nvmoe_ffn_args* args, FfnParams& P) {
    if (!args || !args->pool || !args->x || !args->slot_ids || !args->weights || !args->y)
        return NVMOE_ERR_INVALID_ARG;
    const nvmoe_expert_pool& pool = *args->pool;
    if (!pool_ok(pool)) return NVMOE_ERR_INVALID_ARG;
    if (args->n_tok < 0 || args->top_k <= 0) return NVMOE_ERR_INVALID_ARG;
    const int H = pool.hidden, I = pool.inter;
    if (args->shared) {
        const nvmoe_expert_pool& sp = *args->shared;
        if (!pool_ok(sp) || sp.quant != pool.quant || sp.hidden != H || sp.inter != I)
            return NVMOE_ERR_INVALID_ARG;
    }
    if (pool.quant != NVMOE_Q_NVFP4) return NVMOE_ERR_UNSUPPORTED;
    // warp tiling: gate_up K = H over 8 warps, down K = I per warp, 16-row tiles
    if (H % (kConsumerWarps * FmtNvfp4::kWarpTileK) != 0 || I % FmtNvfp4::kWarpTileK != 0 ||
        I % 16 != 0 || H % 16 != 0)
        return NVMOE_ERR_UNSUPPORTED;
    if (!pool.gate.scale || !pool.up.scale || !pool.down.scale) return NVMOE_ERR_INVALID_ARG;
    if (!pool_aligned(pool) || (args->shared && !pool_aligned(*args->shared)))
        return NVMOE_ERR_INVALID_ARG;
    if (pool.gate.row_stride < H / 2 || pool.down.row_stride < I / 2 ||
        pool.gate.scale_row_stride < H / 16 || pool.down.scale_row_stride < I / 16)
        return NVMOE_ERR_INVALID_ARG;
    if (args->x_row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(args->x) & 15))
        return NVMOE_ERR_INVALID_ARG;
    const WsLayout L = ws_layout(args->n_tok > 0 ? args->n_tok : 1, args->top_k, H, I, pool.n_slots);
    if (!args->workspace || args->workspace_bytes < L.total ||
        (reinterpret_cast<uintptr_t>(args->workspace) & 255))
        return NVMOE_ERR_WORKSPACE;
    P = FfnParams{};
    P.pool = pool;
    P.has_shared = args->shared ? 1 : 0;
    P.shared = args->shared ? *args->shared : pool;
    P.shared_gate = args->shared ? args->shared_gate : nullptr;
    P.x = args->x;
    P.x_stride = args->x_row_stride;
    P.ids = args->slot_ids;
    P.ids_stride = args->ids_row_stride;
    P.w = args->weights;
    P.w_stride = args->weights_row_stride;
    P.top_k = args->top_k;
    P.n_tok = args->n_tok;
    P.y = args->y;
    P.y_stride = args->y_row_stride;
    P.ws = static_cast<unsigned char*>(args->workspace);
    P.L = L;
    P.status = args->status;
    return NVMOE_OK;
}

int ffn_launch_main(FfnParams& P, cudaStream_t st) { return launch_fmt<FmtNvfp4>(P, st); }

int ffn_launch_prep(FfnParams& P, cudaStream_t st) {
    const size_t prep_smem = (size_t)P.pool.n_slots * 4;
    if (prep_smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
    if (prep_smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_prep_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)prep_smem));
    const int conv_blocks = std::min(P.n_tok, 2 * kNumSMs);
    cudaError_t e = launch_pdl(ffn_prep_kernel, dim3(conv_blocks + 1), dim3(kPrepThreads),
                               prep_smem, st, true, P);
    return cuda_status("ffn_prep launch", e);
}

}  // namespace nvmoe

extern "C" size_t nvmoe_moe_ffn_workspace_size(int n_tok, int top_k, int hidden, int inter,
                                               int n_slots) {
    if (n_tok <= 0 || top_k <= 0 || hidden <= 0 || inter <= 0 || n_slots <= 0) return 0;
    return nvmoe::ws_layout(n_tok, top_k, hidden, inter, n_slots).total;
}

extern "C" int nvmoe_moe_ffn(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    FfnParams P;
    const int rc = ffn_setup(args, P);
    if (rc != NVMOE_OK) return rc;
    if (args->n_tok == 0) return NVMOE_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int r1 = ffn_launch_prep(P, st);
    if (r1 != NVMOE_OK) return r1;
    return ffn_launch_main(P, st);
}
