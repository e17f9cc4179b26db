// R1 — router top-k over fp32 logits, one warp per token row.
//
// Reference behaviour:
//   softmax -> argsort top-k -> get_rows -> sum/div renormalisation (llama.cpp build_moe_ffn as
//   exercised by scripts/test_sched_chain_shrink.cpp:108-121);
//   GLM: sigmoid(logits) + e_score_correction_bias for the choice, weights gathered from the
//   plain sigmoid scores, normalised by (sum + 1e-20), times routed_scaling_factor
//   (nvme-moe-bench/nvme_offload_cache.py:3044-3089).
//
// Selection is an exact k-pass arg-max over a per-lane register tile: the key order is a
// strict total order (key descending, then expert id ascending), so the chosen ids do not
// depend on thread scheduling.  Softmax selection uses the logits themselves (softmax is
// monotone), so ties between distinct logits cannot be introduced by exp rounding.
#include "common.cuh"

namespace nvmoe {
namespace {

constexpr int kMaxExperts = 1024;
constexpr int kPerLane = kMaxExperts / 32;
constexpr int kMaxTopK = 32;

__device__ __forceinline__ bool key_better(float ka, int ia, float kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

__global__ void __launch_bounds__(256) router_topk_kernel(
    const float* __restrict__ logits, int64_t lstride, int n_tok, int n_expert, int top_k,
    int mode, const float* __restrict__ bias, int norm_topk, float scaling,
    int32_t* __restrict__ out_ids, int64_t istride, float* __restrict__ out_w, int64_t wstride) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n_tok) return;
    const float* lr = logits + (int64_t)row * lstride;

    float key[kPerLane];
    float val[kPerLane];  // softmax: logit; sigmoid: score
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int e = i * 32 + lane;
        float k = -INFINITY, v = -INFINITY;
        if (e < n_expert) {
            float l = lr[e];
            if (mode == NVMOE_ROUTER_SOFTMAX) {
                v = l;
                k = (l != l) ? -INFINITY : l;  // NaN logits never win
            } else {
                float s = 1.0f / (1.0f + expf(-l));
                v = s;
                float c = s + (bias ? bias[e] : 0.0f);
                k = (c != c) ? -INFINITY : c;
            }
        }
        key[i] = k;
        val[i] = v;
    }

    // Lane j keeps the j-th pick (top_k <= 32), so no per-thread arrays spill to local memory.
    float my_val = 0.f, first_val = 0.f;
    int my_id = -1;
    uint32_t taken = 0;  // bit i: expert i*32+lane already chosen
    for (int j = 0; j < top_k; ++j) {
        float bk = -INFINITY;
        int bi = 0x7fffffff;
        float bv = 0.f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int e = i * 32 + lane;
            if (e < n_expert && !((taken >> i) & 1u) && key_better(key[i], e, bk, bi)) {
                bk = key[i];
                bi = e;
                bv = val[i];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ok = __shfl_xor_sync(0xffffffffu, bk, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            if (key_better(ok, oi, bk, bi)) {
                bk = ok;
                bi = oi;
                bv = ov;
            }
        }
        if (lane == j) my_id = bi, my_val = bv;
        if (j == 0) first_val = bv;
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    }

    // Full-softmax denominator (only when the top-k weights are not renormalised).
    float full_denom = 0.f;
    if (mode == NVMOE_ROUTER_SOFTMAX && !norm_topk) {
        const float m = first_val;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int e = i * 32 + lane;
            if (e < n_expert && val[i] == val[i]) full_denom += expf(val[i] - m);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) full_denom += __shfl_xor_sync(0xffffffffu, full_denom, o);
    }

    const bool mine = lane < top_k;
    float w;
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        // probabilities relative to the row maximum (= the first pick)
        w = mine ? expf(my_val - first_val) : 0.f;
    } else {
        w = mine ? my_val : 0.f;
    }
    // sum of the picks in pick order (lane 0 first), identical on every lane
    float sum = 0.f;
    for (int j = 0; j < top_k; ++j) sum += __shfl_sync(0xffffffffu, w, j);
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        const float denom = norm_topk ? sum : full_denom;
        w = w / denom * scaling;
    } else {
        w = (norm_topk ? w / (sum + 1e-20f) : w) * scaling;
    }
    if (mine) {
        out_ids[(int64_t)row * istride + lane] = my_id;
        out_w[(int64_t)row * wstride + lane] = w;
    }
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_router_topk(const float* logits, int64_t logits_row_stride, int n_tok,
                                 int n_expert, int top_k, int mode, const float* bias,
                                 int norm_topk, float routed_scaling, int32_t* out_ids,
                                 int64_t ids_row_stride, float* out_weights,
                                 int64_t weights_row_stride, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (n_tok < 0 || n_expert <= 0 || n_expert > kMaxExperts || top_k <= 0 ||
        top_k > kMaxTopK || top_k > n_expert)
        return NVMOE_ERR_INVALID_ARG;
    if (mode != NVMOE_ROUTER_SOFTMAX && mode != NVMOE_ROUTER_SIGMOID_BIAS)
        return NVMOE_ERR_INVALID_ARG;
    if (n_tok == 0) return NVMOE_OK;
    if (!logits || !out_ids || !out_weights) return NVMOE_ERR_INVALID_ARG;
    const int warps = 8;
    dim3 grid((n_tok + warps - 1) / warps), block(32 * warps);
    router_topk_kernel<<<grid, block, 0, (cudaStream_t)stream>>>(
        logits, logits_row_stride, n_tok, n_expert, top_k, mode, bias, norm_topk, routed_scaling,
        out_ids, ids_row_stride, out_weights, weights_row_stride);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}
