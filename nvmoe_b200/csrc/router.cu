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
#include "router_device.cuh"

namespace nvmoe {
namespace {

__global__ void __launch_bounds__(256) router_topk_kernel(
    const float* __restrict__ logits, int64_t lstride, int n_tok, int n_expert, int top_k,
    int mode, const float* __restrict__ bias, int norm_topk, float scaling,
    int32_t* __restrict__ out_ids, int64_t istride, float* __restrict__ out_w, int64_t wstride) {
    const int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (row >= n_tok) return;
    router_topk_warp(logits + (int64_t)row * lstride, n_expert, top_k, mode, bias, norm_topk,
                     scaling, out_ids + (int64_t)row * istride, out_w + (int64_t)row * wstride);
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
