// One decode layer step (engine path): fused router + remap + FFN grouping kernel, then the
// optional refill gather and the FFN kernels, all chained with programmatic dependent launch.
//
// The front kernel is one CTA of 512 threads: warps compute the top-k of the token rows
// (router_device.cuh), the block then runs the remap (remap_device.cuh) in place on the ids and
// groups the slot ids for the FFN (ffn_common.cuh).  Replaces three launches (router, remap,
// FFN prep) on the latency-critical small-batch decode path.
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

constexpr int kFrontThreads = 512;  // 16 warps; 128 registers per thread for the top-k tile

struct FrontParams {
    const float* logits;
    int64_t lstride;
    int mode;
    const float* bias;
    int norm_topk;
    float scaling;
    RemapParams rp;
    float* weights;
    FfnParams fp;
};

__global__ void __launch_bounds__(kFrontThreads, 1) decode_front_kernel(FrontParams F) {
    extern __shared__ __align__(16) unsigned char smem[];
    grid_dep_wait();
    grid_dep_launch();
    const int warp = threadIdx.x >> 5, nw = blockDim.x >> 5;
    const int k = F.rp.top_k;
    int32_t* ids = F.rp.out;
    for (int t = warp; t < F.rp.n_tok; t += nw)
        router_topk_warp(F.logits + (int64_t)t * F.lstride, F.rp.t.n_expert, k, F.mode, F.bias,
                         F.norm_topk, F.scaling, ids + (int64_t)t * k, F.weights + (int64_t)t * k);
    __syncthreads();
    const int st = remap_block(F.rp, smem);
    ffn_convert_tokens(F.fp, 0, 1);
    if (st != NVMOE_OK) {  // ids were not rewritten: give the FFN nothing to do (y = 0)
        if (threadIdx.x == 0) {
            int* hdr = wsp<int>(F.fp, F.fp.L.hdr);
            hdr[HDR_N_GROUPS] = 0;
            hdr[HDR_N_ACTIVE] = 0;
            hdr[HDR_N_ENT] = 0;
            hdr[HDR_STATUS] = st;
            if (F.fp.status) *F.fp.status = st;
        }
        return;
    }
    ffn_group_block(F.fp, reinterpret_cast<int*>(smem));
}

}  // namespace

int ffn_launch_main(FfnParams& P, cudaStream_t st);
int ffn_setup(const nvmoe_ffn_args* args, FfnParams& P);

}  // namespace nvmoe

extern "C" int nvmoe_decode_layer(const nvmoe_decode_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->logits || !a->slot_ids || !a->weights) return NVMOE_ERR_INVALID_ARG;
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

    const size_t smem = std::max(remap_smem_bytes(t.n_expert, t.cache_size),
                                 (size_t)F.fp.pool.n_slots * 4);
    if (smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
    cudaStream_t st = (cudaStream_t)stream;
    if (smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(decode_front_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    cudaError_t e = launch_pdl(decode_front_kernel, dim3(1), dim3(kFrontThreads), smem, st, true, F);
    if (e != cudaSuccess) return cuda_status("decode_front launch", e);
    if (a->refill_banks && a->n_refill_banks > 0) {
        rc = nvmoe_refill_gather(a->refill_banks, a->n_refill_banks, &a->misses,
                                 a->host_slot_of_id, t.cache_size, stream);
        if (rc != NVMOE_OK) return rc;
    }
    return ffn_launch_main(F.fp, st);
}
