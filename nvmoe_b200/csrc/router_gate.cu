// In front of the router top-k in a decoder stack: residual add, RMSNorm and the router gate
// GEMV of one MoE layer, in one launch (nvmoe_router_gate).
//
// Reference: Qwen4ExpMoE.forward runs gate.forward(hidden) on the normalised hidden state
// (nvme-moe-bench/nvme_offload_cache.py:2114) to produce the router logits that the cache hook's
// top-k and slot remap consume; the decoder layer in front of it adds the residual and applies
// RMSNorm.  FreeToken (which holds those modules) is not in the reference tree; the arithmetic
// here is the usual decoder-layer form:
//   h      = bf16(resid + delta)                                  (fp32 add, one rounding)
//   x      = bf16(gamma * bf16(h * (1 / sqrt(mean(h^2) + eps))))  (RMSNorm, fp32 statistics)
//   logits = x . W_gate^T (+ logit_bias)                          (fp32 accumulation)
//
// Layout: a 2-D grid of CTAs, one per (block of kGateRows gate rows, block of kGateTok tokens),
// 8 warps each.  Warps w and w + 4 hold gate row w of the block in registers, loaded before the
// dependency wait (the weights are constant, so their load overlaps the previous kernel's
// tail).  After the wait each warp normalises one token of the block into shared memory (CTAs
// of the first row block also store h and x); then warp w dots its row with the block's tokens
// of parity w / 4, two tokens at a time.  The gate matrix is read from HBM once; the token rows
// are re-read from L2 by each row block.  With the fused top-k, each CTA counts itself done on
// its token block (fence, then a ticket); the last one routes the block's tokens, a warp each.
#include "common.cuh"
#include "router_device.cuh"

#include <algorithm>

namespace nvmoe {
namespace {

constexpr int kGateRows = 4;   // gate rows per CTA (each held by two warps)
constexpr int kGateTok = 8;    // tokens per CTA (one per warp in the normalisation)
constexpr int kGateWarps = 8;
constexpr int kGateThreads = 32 * kGateWarps;

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
    return (uint32_t)f32_to_bf16_bits(lo) | ((uint32_t)f32_to_bf16_bits(hi) << 16);
}
__device__ __forceinline__ float bf16_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

// NCH = H / 256: a lane holds 8 values (16 bytes of bf16) of each 256-wide chunk of a row.
template <int NCH>
__global__ void __launch_bounds__(kGateThreads) router_gate_kernel(nvmoe_router_gate_args a) {
    extern __shared__ __align__(16) unsigned char smem[];
    uint4* xs = reinterpret_cast<uint4*>(smem);  // [kGateTok][H / 8] normalised tokens
    constexpr int H = NCH * 256;
    constexpr int VPR = H / 8;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int e = blockIdx.x * kGateRows + (warp & (kGateRows - 1));
    const bool has_row = a.gate_weight && e < a.n_expert;
    const int t0 = blockIdx.y * kGateTok;
    const int nt = min(kGateTok, a.n_tok - t0);
    uint4 w[NCH];
    if (has_row) {
        const uint16_t* wr = a.gate_weight + (int64_t)e * a.gate_row_stride;
#pragma unroll
        for (int c = 0; c < NCH; ++c) w[c] = ldg_stream16(wr + c * 256 + lane * 8);
    }
    grid_dep_launch();
    grid_dep_wait();  // the residual / delta rows come from the kernel before this one

    const bool writer = blockIdx.x == 0;
    for (int i = warp; i < nt; i += kGateWarps) {
        const int t = t0 + i;
        const uint16_t* rr = a.resid + (int64_t)t * a.resid_row_stride;
        const uint16_t* dr = a.delta ? a.delta + (int64_t)t * a.delta_row_stride : nullptr;
        uint32_t hv[NCH][4];
        uint4 rv[NCH], dv[NCH];
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            rv[c] = *reinterpret_cast<const uint4*>(rr + c * 256 + lane * 8);
            dv[c] = dr ? *reinterpret_cast<const uint4*>(dr + c * 256 + lane * 8)
                       : make_uint4(0, 0, 0, 0);
        }
        float ssp[4] = {0.f, 0.f, 0.f, 0.f};  // four chains, summed in a fixed order below
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            float& ss = ssp[c & 3];
            const uint32_t* r4 = reinterpret_cast<const uint32_t*>(&rv[c]);
            const uint32_t* d4 = reinterpret_cast<const uint32_t*>(&dv[c]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if (dr) {
                    const float lo = __fadd_rn(bf16_lo(r4[q]), bf16_lo(d4[q]));
                    const float hi = __fadd_rn(bf16_hi(r4[q]), bf16_hi(d4[q]));
                    hv[c][q] = pack_bf16x2(lo, hi);
                } else {
                    hv[c][q] = r4[q];  // h = resid as given (keeps -0)
                }
                const float l2 = bf16_lo(hv[c][q]), h2 = bf16_hi(hv[c][q]);
                ss = __fmaf_rn(l2, l2, ss);
                ss = __fmaf_rn(h2, h2, ss);
            }
        }
        float ss = (ssp[0] + ssp[1]) + (ssp[2] + ssp[3]);
        if (writer && a.resid_out) {
            uint16_t* o = a.resid_out + (int64_t)t * a.resid_out_row_stride;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
                *reinterpret_cast<uint4*>(o + c * 256 + lane * 8) =
                    make_uint4(hv[c][0], hv[c][1], hv[c][2], hv[c][3]);
        }
        if (a.norm_weight) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            const float inv =
                __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)H), a.eps)));
#pragma unroll
            for (int c = 0; c < NCH; ++c) {
                const uint4 gv = *reinterpret_cast<const uint4*>(a.norm_weight + c * 256 + lane * 8);
                const uint32_t* g4 = reinterpret_cast<const uint32_t*>(&gv);
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t n = pack_bf16x2(__fmul_rn(bf16_lo(hv[c][q]), inv),
                                                   __fmul_rn(bf16_hi(hv[c][q]), inv));
                    hv[c][q] = pack_bf16x2(__fmul_rn(bf16_lo(g4[q]), bf16_lo(n)),
                                           __fmul_rn(bf16_hi(g4[q]), bf16_hi(n)));
                }
            }
        }
        if (writer && a.x_out) {
            uint16_t* o = a.x_out + (int64_t)t * a.x_out_row_stride;
#pragma unroll
            for (int c = 0; c < NCH; ++c)
                *reinterpret_cast<uint4*>(o + c * 256 + lane * 8) =
                    make_uint4(hv[c][0], hv[c][1], hv[c][2], hv[c][3]);
        }
#pragma unroll
        for (int c = 0; c < NCH; ++c)
            xs[i * VPR + c * 32 + lane] = make_uint4(hv[c][0], hv[c][1], hv[c][2], hv[c][3]);
    }
    if (!a.gate_weight) return;
    __syncthreads();
    // tokens of this warp's parity, two at a time (four independent accumulation chains)
    for (int i = warp >> 2; has_row && i < nt; i += 4) {
        const int i2 = i + 2 < nt ? i + 2 : i;
        float acc[2][2] = {{0.f, 0.f}, {0.f, 0.f}};
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
            const uint4 xv0 = xs[i * VPR + c * 32 + lane];
            const uint4 xv1 = xs[i2 * VPR + c * 32 + lane];
            const uint32_t* x0 = reinterpret_cast<const uint32_t*>(&xv0);
            const uint32_t* x1 = reinterpret_cast<const uint32_t*>(&xv1);
            const uint32_t* w4 = reinterpret_cast<const uint32_t*>(&w[c]);
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                acc[0][q & 1] = __fmaf_rn(bf16_lo(x0[q]), bf16_lo(w4[q]), acc[0][q & 1]);
                acc[0][q & 1] = __fmaf_rn(bf16_hi(x0[q]), bf16_hi(w4[q]), acc[0][q & 1]);
                acc[1][q & 1] = __fmaf_rn(bf16_lo(x1[q]), bf16_lo(w4[q]), acc[1][q & 1]);
                acc[1][q & 1] = __fmaf_rn(bf16_hi(x1[q]), bf16_hi(w4[q]), acc[1][q & 1]);
            }
        }
        float r0 = acc[0][0] + acc[0][1], r1 = acc[1][0] + acc[1][1];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            r0 += __shfl_xor_sync(0xffffffffu, r0, o);
            r1 += __shfl_xor_sync(0xffffffffu, r1, o);
        }
        if (lane == 0) {
            const float b = a.logit_bias ? a.logit_bias[e] : 0.f;
            a.logits[(int64_t)(t0 + i) * a.logits_row_stride + e] =
                a.logit_bias ? __fadd_rn(r0, b) : r0;
            if (i2 != i)
                a.logits[(int64_t)(t0 + i2) * a.logits_row_stride + e] =
                    a.logit_bias ? __fadd_rn(r1, b) : r1;
        }
    }
    if (a.top_k <= 0) return;
    // fused top-k: the last CTA done on this token block routes it
    __shared__ int s_last;
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const int done = atomicAdd(a.tickets + blockIdx.y, 1);
        s_last = done == (int)gridDim.x - 1;
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    for (int i = warp; i < nt; i += kGateWarps) {
        const int t = t0 + i;
        router_topk_warp(a.logits + (int64_t)t * a.logits_row_stride, a.n_expert, a.top_k,
                         a.router_mode, a.router_bias, a.norm_topk, a.routed_scaling,
                         a.out_ids + (int64_t)t * a.top_k, a.out_weights + (int64_t)t * a.top_k);
    }
    if (threadIdx.x == 0) a.tickets[blockIdx.y] = 0;  // ready for the next call
}

template <int NCH>
int launch_gate(const nvmoe_router_gate_args& a, dim3 grid, cudaStream_t st) {
    const size_t smem = (size_t)kGateTok * NCH * 256 * 2;
    if (smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(router_gate_kernel<NCH>,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const cudaError_t e =
        launch_pdl(router_gate_kernel<NCH>, grid, dim3(kGateThreads), smem, st, true, a);
    return cuda_status("router_gate launch", e);
}

bool overlaps(const void* a, int64_t a_bytes, const void* b, int64_t b_bytes) {
    if (!a || !b) return false;
    const uintptr_t x = reinterpret_cast<uintptr_t>(a), y = reinterpret_cast<uintptr_t>(b);
    return x < y + (uintptr_t)b_bytes && y < x + (uintptr_t)a_bytes;
}

bool rows_ok(const void* p, int64_t stride) {
    return !p || ((reinterpret_cast<uintptr_t>(p) & 15) == 0 && stride % 8 == 0);
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_router_gate(const nvmoe_router_gate_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->resid || a->n_tok < 0) return NVMOE_ERR_INVALID_ARG;
    const int H = a->hidden;
    if (H != 1024 && H != 2048 && H != 4096) return NVMOE_ERR_UNSUPPORTED;
    if (a->gate_weight && (!a->logits || a->n_expert <= 0)) return NVMOE_ERR_INVALID_ARG;
    if (!rows_ok(a->resid, a->resid_row_stride) || !rows_ok(a->delta, a->delta_row_stride) ||
        !rows_ok(a->resid_out, a->resid_out_row_stride) ||
        !rows_ok(a->x_out, a->x_out_row_stride) || !rows_ok(a->gate_weight, a->gate_row_stride) ||
        !rows_ok(a->norm_weight, 0))
        return NVMOE_ERR_INVALID_ARG;
    if (a->top_k > 0 &&
        (!a->gate_weight || a->top_k > kMaxTopK || a->top_k > a->n_expert ||
         a->n_expert > kMaxExperts || !a->out_ids || !a->out_weights || !a->tickets ||
         (a->router_mode != NVMOE_ROUTER_SOFTMAX && a->router_mode != NVMOE_ROUTER_SIGMOID_BIAS)))
        return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok == 0) return NVMOE_OK;
    // every CTA reads resid / delta while CTA 0 writes resid_out and x_out: no overlap allowed
    const int64_t rb = ((int64_t)(a->n_tok - 1) * std::max<int64_t>(a->resid_row_stride, 0) + H) * 2;
    const int64_t db = ((int64_t)(a->n_tok - 1) * std::max<int64_t>(a->delta_row_stride, 0) + H) * 2;
    const int64_t ob = ((int64_t)(a->n_tok - 1) * std::max<int64_t>(a->resid_out_row_stride, 0) + H) * 2;
    const int64_t xb = ((int64_t)(a->n_tok - 1) * std::max<int64_t>(a->x_out_row_stride, 0) + H) * 2;
    for (const auto& w : {std::make_pair((const void*)a->resid_out, ob),
                          std::make_pair((const void*)a->x_out, xb)})
        if (overlaps(w.first, w.second, a->resid, rb) || overlaps(w.first, w.second, a->delta, db))
            return NVMOE_ERR_INVALID_ARG;
    const dim3 grid(a->gate_weight ? (a->n_expert + kGateRows - 1) / kGateRows : 1,
                    (a->n_tok + kGateTok - 1) / kGateTok);
    if (grid.y > 65535) return NVMOE_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream;
    switch (H / 256) {
        case 4: return launch_gate<4>(*a, grid, st);
        case 8: return launch_gate<8>(*a, grid, st);
        default: return launch_gate<16>(*a, grid, st);
    }
}
