// Cache counters: eval_cb's statistics (scripts/moe_cache_probe.cpp:253-256, updated per
// distinct id at :662-671 and per call at :995), accumulated on the device from the miss list
// a remap or decode layer step wrote, so no count crosses to the host during a step.
#include "common.cuh"

namespace nvmoe {
namespace {

__global__ void cache_stats_add_kernel(nvmoe_cache_stats* s, const int32_t* counts, int is_decode,
                                       int64_t bytes_per_expert) {
    if (threadIdx.x != 0) return;
    const int nu = counts[0], nm = counts[1], status = counts[2];
    using ull = unsigned long long;
    if (status != NVMOE_OK || nu < 0 || nm < 0 || nm > nu) {
        atomicAdd(reinterpret_cast<ull*>(&s->error_calls), 1ull);
        return;
    }
    // (atomics: calls on several streams may add to the same counters)
    atomicAdd(reinterpret_cast<ull*>(&s->calls), 1ull);
    atomicAdd(reinterpret_cast<ull*>(&s->gpu_hits), (ull)(nu - nm));
    atomicAdd(reinterpret_cast<ull*>(&s->gpu_misses), (ull)nm);
    atomicAdd(reinterpret_cast<ull*>(&s->refill_bytes), (ull)((int64_t)nm * bytes_per_expert));
    if (is_decode) {
        atomicAdd(reinterpret_cast<ull*>(&s->decode_calls), 1ull);
        atomicAdd(reinterpret_cast<ull*>(&s->decode_gpu_hits), (ull)(nu - nm));
        atomicAdd(reinterpret_cast<ull*>(&s->decode_gpu_misses), (ull)nm);
    }
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_cache_stats_add(nvmoe_cache_stats* stats, const int32_t* counts,
                                     int is_decode, int64_t bytes_per_expert,
                                     nvmoe_stream_t stream) {
    if (!stats || !counts || bytes_per_expert < 0) return NVMOE_ERR_INVALID_ARG;
    if ((reinterpret_cast<uintptr_t>(stats) & 7) || (reinterpret_cast<uintptr_t>(counts) & 3))
        return NVMOE_ERR_INVALID_ARG;
    nvmoe::cache_stats_add_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(stats, counts, is_decode,
                                                                     bytes_per_expert);
    return nvmoe::cuda_status("cache_stats_add launch", cudaGetLastError());
}
