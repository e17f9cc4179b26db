// (f)3 tail pruning on the device (scripts/moe_cache_probe.cpp:523-625): one thread per token
// row runs prune_row (prune_device.cuh) on the row's ids and router weights in place, between
// the router top-k and the slot remap, so pruned picks alias a resident expert and cost no copy.
// The reference reads the weights back to the host for this; here nothing leaves the device.
#include "common.cuh"
#include "prune_device.cuh"

namespace nvmoe {
namespace {

constexpr int kPruneThreads = 128;

__global__ void __launch_bounds__(kPruneThreads) prune_kernel(nvmoe_prune_args a, PruneCfg c) {
    const int t = blockIdx.x * kPruneThreads + threadIdx.x;
    if (t >= a.n_tok) return;
    // the expert of the pool's first occupied slot (the reference's alias of last resort)
    int32_t resident_real = -1;
    for (int s = 0; s < a.cache_size && resident_real == -1; ++s) resident_real = a.real_in_slot[s];
    if (resident_real == -1) return;
    int32_t* ids = a.ids + (int64_t)t * a.ids_row_stride;
    float* w = a.weights + (int64_t)t * a.weights_row_stride;
    for (int i = 0; i < a.top_k; ++i)  // ids outside the tables: the row is left as it is
        if (ids[i] < 0 || ids[i] >= a.n_expert) return;
    int pruned[2] = {0, 0};
    prune_row(ids, w, a.top_k, a.slot_of_real, a.host_slot_of_real, resident_real, c, pruned);
    if (a.pruned && a.is_decode) {
        if (pruned[0]) atomicAdd(a.pruned, pruned[0]);
        if (pruned[1]) atomicAdd(a.pruned + 1, pruned[1]);
    }
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_prune_tail(const nvmoe_prune_args* a, nvmoe_stream_t stream) {
    if (!a || a->n_tok < 0 || a->top_k <= 0 || a->top_k > 32 || a->n_expert <= 0 ||
        a->cache_size <= 0 || a->min_keep < 0)
        return NVMOE_ERR_INVALID_ARG;
    if (!a->ids || !a->weights || !a->slot_of_real || !a->real_in_slot ||
        a->ids_row_stride < a->top_k || a->weights_row_stride < a->top_k)
        return NVMOE_ERR_INVALID_ARG;
    // the reference prunes only with a backing-store threshold set and at most 4096 picks
    if (!(a->nvme_thresh > 0.0f) || (int64_t)a->n_tok * a->top_k > 4096 || a->n_tok == 0)
        return NVMOE_OK;
    nvmoe::PruneCfg c{a->nvme_thresh, a->host_thresh, a->min_mass, a->min_keep};
    const int blocks = (a->n_tok + nvmoe::kPruneThreads - 1) / nvmoe::kPruneThreads;
    nvmoe::prune_kernel<<<blocks, nvmoe::kPruneThreads, 0, (cudaStream_t)stream>>>(*a, c);
    return nvmoe::cuda_status("prune_tail launch", cudaGetLastError());
}
