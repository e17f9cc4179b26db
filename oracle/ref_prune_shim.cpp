// Test infrastructure (never linked into the product): the reference's own decode-time tail
// pruning, compiled from scripts/moe_cache_probe.cpp itself.  oracle/Makefile extracts its lines
// 523-625 (the "two-tier cost-aware expert pruning" block of eval_cb) into oracle/_ref/ and this
// file compiles them inside one function, with stand-ins for what the block names: the layer's
// residency tables (layer_cache, moe_cache_probe.cpp:207-247), the pruning settings and counters
// (cache_state, :253-272), the router-weights tensor (t->data with its row stride t->nb[2]) and
// the CUDA copies between it and the pinned staging rows (host memcpy here).
#include <cstdint>
#include <cstring>
#include <vector>

namespace {

enum { cudaMemcpyDeviceToHost = 2, cudaMemcpyHostToDevice = 1 };
void* const cudaStreamPerThread = nullptr;
inline int cudaMemcpy(void* d, const void* s, size_t n, int) {
    std::memcpy(d, s, n);
    return 0;
}
inline int cudaMemcpyAsync(void* d, const void* s, size_t n, int, void*) {
    std::memcpy(d, s, n);
    return 0;
}

struct layer_cache_stub {
    int64_t cache_size = 0;
    std::vector<int32_t> slot_of_real, real_in_slot, host_slot_of_real;
};
struct cache_state_stub {
    float prune_nvme_thresh = 0.0f, prune_host_thresh = 0.0f, prune_min_mass = 0.95f;
    int prune_min_keep = 6;
    float* pinned_weights = nullptr;
    bool is_decode_phase = true;
    long decode_pruned_nvme = 0, decode_pruned_host = 0;
};
struct tensor_stub {
    void* data = nullptr;
    size_t nb[4] = {0, 0, 0, 0};
};

}  // namespace

// ids [n_tokens][n_expert_used] and weights (same layout) are rewritten in place.
extern "C" void ref_prune(int n_expert, int cache_size, const int32_t* slot_of_real,
                          const int32_t* host_slot_of_real, const int32_t* real_in_slot,
                          int32_t* ids_io, float* weights_io, int n_tokens, int n_expert_used,
                          float nvme_thresh, float host_thresh, int min_keep, float min_mass,
                          int is_decode, long* pruned_nvme, long* pruned_host) {
    layer_cache_stub lc;
    lc.cache_size = cache_size;
    lc.slot_of_real.assign(slot_of_real, slot_of_real + n_expert);
    lc.host_slot_of_real.assign(host_slot_of_real, host_slot_of_real + n_expert);
    lc.real_in_slot.assign(real_in_slot, real_in_slot + cache_size);
    std::vector<float> staging(4096);
    cache_state_stub state;
    state.prune_nvme_thresh = nvme_thresh;
    state.prune_host_thresh = host_thresh;
    state.prune_min_keep = min_keep;
    state.prune_min_mass = min_mass;
    state.pinned_weights = staging.data();
    state.is_decode_phase = is_decode != 0;
    cache_state_stub* st = &state;
    tensor_stub tw;
    tw.data = weights_io;
    tw.nb[2] = sizeof(float) * (size_t)n_expert_used;
    tensor_stub* t = &tw;
    std::vector<int32_t> ids(ids_io, ids_io + (size_t)n_tokens * n_expert_used);
    const int64_t n_tokens_ = n_tokens;
    {
        const int64_t n_tokens = n_tokens_;
        const int64_t n_expert_used_ = n_expert_used;
        const int64_t n_expert_used = n_expert_used_;
#include "prune_block.inc"
    }
    std::memcpy(ids_io, ids.data(), ids.size() * sizeof(int32_t));
    *pruned_nvme = state.decode_pruned_nvme;
    *pruned_host = state.decode_pruned_host;
}
