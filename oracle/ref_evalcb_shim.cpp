// Test infrastructure (never linked into the product): the reference's own eval_cb GPU-tier and
// host-tier block, compiled from scripts/moe_cache_probe.cpp itself.  oracle/Makefile extracts
// its lines 627-753 (distinct ids, hits, GPU victims, host-tier placement) and 955-970 (the ids
// rewritten to slots) into oracle/_ref/ and this file compiles them inside one function, with
// stand-ins for the two structs the block reads (the fields of layer_cache and cache_state it
// names, moe_cache_probe.cpp:207-260) and the reference's own SegmentedHostLru header.  The
// block aborts where the reference aborts (more distinct ids than slots): callers stay within
// the pool.
#include <algorithm>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <unordered_set>
#include <vector>

#include "segmented_host_lru.hpp"

namespace {

struct layer_cache_stub {
    int64_t n_expert_real = 0;
    int64_t cache_size = 0;
    bool fused_gate_up = true;
    std::vector<int32_t> slot_of_real, real_in_slot;
    std::vector<uint32_t> slot_last_used;
    uint32_t current_step = 0;
    int64_t host_cache_size = 0;
    SegmentedHostLru<int32_t> host_lru;
    std::vector<int32_t> host_slot_of_real, host_real_in_slot;
    int32_t host_next_free = 0;
    std::vector<int64_t> access_count;
    int32_t gpu_pinned_k = 0;
    explicit layer_cache_stub(double ratio) : host_lru(ratio) {}
};

struct cache_state_stub {
    bool is_decode_phase = false;
    long hits = 0, misses = 0, host_hits = 0, host_misses = 0;
    long decode_hits = 0, decode_misses = 0, decode_host_hits = 0, decode_host_misses = 0;
};

struct handle {
    layer_cache_stub lc;
    cache_state_stub st;
    explicit handle(double r) : lc(r) {}
};

}  // namespace

extern "C" void* ref_evalcb_create(int n_expert, int cache_size, int pinned_k, int host_cache_size,
                                   double protected_ratio) {
    handle* h = new handle(protected_ratio);
    layer_cache_stub& lc = h->lc;
    lc.n_expert_real = n_expert;
    lc.cache_size = cache_size;
    lc.slot_of_real.assign((size_t)n_expert, -1);
    lc.real_in_slot.assign((size_t)cache_size, -1);
    lc.slot_last_used.assign((size_t)cache_size, 0);
    lc.host_cache_size = host_cache_size;
    lc.host_lru.set_capacity_hint(host_cache_size);
    lc.host_slot_of_real.assign((size_t)n_expert, -1);
    lc.host_real_in_slot.assign((size_t)(host_cache_size > 0 ? host_cache_size : 1), -1);
    lc.access_count.assign((size_t)n_expert, 0);
    lc.gpu_pinned_k = pinned_k;
    return h;
}

extern "C" void ref_evalcb_destroy(void* p) { delete static_cast<handle*>(p); }

// One eval_cb step for the routed ids [n_tokens, n_expert_used] (contiguous): out_slots gets the
// rewritten ids; the host-tier work of the step comes out as h2d (gpu slot, host slot) pairs for
// host hits and (id, gpu slot, host slot) loads for host misses, in the block's order.
extern "C" int ref_evalcb_step(void* p, const int32_t* ids_in, int n_tokens_in, int n_used_in,
                               int is_decode, int32_t* out_slots, int32_t* h2d_gpu,
                               int32_t* h2d_host, int32_t* n_h2d, int32_t* load_ids,
                               int32_t* load_gpu, int32_t* load_host, int32_t* n_load) {
    handle* h = static_cast<handle*>(p);
    layer_cache_stub& lc = h->lc;
    cache_state_stub* st = &h->st;
    st->is_decode_phase = is_decode != 0;
    const int il = 0;
    const int64_t n_expert_used = n_used_in;
    const int64_t n_tokens = n_tokens_in;
    const int64_t n = n_expert_used * n_tokens;
    std::vector<int32_t> ids(ids_in, ids_in + n);
#include "evalcb_block.inc"
#include "evalcb_rewrite.inc"
    (void)any_gpu_fill;
    std::memcpy(out_slots, ids.data(), sizeof(int32_t) * (size_t)n);
    *n_h2d = (int32_t)host_hits_to_transfer.size();
    for (size_t i = 0; i < host_hits_to_transfer.size(); ++i) {
        h2d_gpu[i] = host_hits_to_transfer[i].gpu_slot;
        h2d_host[i] = host_hits_to_transfer[i].host_slot;
    }
    *n_load = (int32_t)nvme_tasks.size();
    for (size_t i = 0; i < nvme_tasks.size(); ++i) {
        load_ids[i] = nvme_tasks[i].real_id;
        load_gpu[i] = nvme_tasks[i].gpu_slot;
        load_host[i] = nvme_tasks[i].host_slot;
    }
    return 0;
}

extern "C" void ref_evalcb_tables(void* p, int32_t* slot_of_real, int32_t* real_in_slot,
                                  uint32_t* slot_last_used, uint32_t* current_step) {
    const layer_cache_stub& lc = static_cast<handle*>(p)->lc;
    std::copy(lc.slot_of_real.begin(), lc.slot_of_real.end(), slot_of_real);
    std::copy(lc.real_in_slot.begin(), lc.real_in_slot.end(), real_in_slot);
    std::copy(lc.slot_last_used.begin(), lc.slot_last_used.end(), slot_last_used);
    *current_step = lc.current_step;
}
