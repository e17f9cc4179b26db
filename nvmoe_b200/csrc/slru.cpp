// R4 — segmented LRU (2Q / SLRU) policy of the pinned host tier.
//
// Behaviour follows the reference policy (nvme-moe-bench/nvme_offload_cache.py:333-409 and its
// C++ counterpart scripts/segmented_host_lru.hpp:85-160):
//   - insert_new puts a key at the MRU end of `probation` (first reference);
//   - touch promotes probation -> protected (second reference), demoting protected's LRU key
//     back to probation's MRU end when protected is at cap = max(1, floor(capacity * ratio));
//     a key already protected is refreshed; unknown keys are ignored;
//   - pop_lru drains probation's LRU end first, then protected's;
//   - pop_lru_excluding skips protected keys (probation first, then protected) and falls back to
//     pop_lru when every key is excluded;
//   - the first capacity hint wins; without one there is no protected cap.
// Implementation: one slab of nodes (reused through a free list) in two intrusive doubly-linked
// lists, indexed by a std::unordered_map from key to node.  Operations are O(1) on average; an
// insert of a new key may allocate a hash node, and pop_lru_excluding builds a hash set of the
// excluded keys on each call.
#include <algorithm>
#include <cstdint>
#include <cstdlib>
#include <unordered_map>
#include <unordered_set>
#include <vector>
#include <cmath>

#include "../../include/nvmoe_b200.h"

namespace nvmoe {

class SegmentedLru {
   public:
    explicit SegmentedLru(double ratio) : ratio_(ratio) {
        for (int s = 0; s < 2; ++s) head_[s] = tail_[s] = -1, size_[s] = 0;
    }

    bool contains(int64_t k) const { return index_.count(k) != 0; }
    int64_t size() const { return size_[0] + size_[1]; }

    void set_capacity_hint(int64_t c) {
        if (!has_cap_) {
            has_cap_ = true;
            cap_ = c;
        }
    }

    void insert_new(int64_t k) {
        auto it = index_.find(k);
        if (it != index_.end()) unlink(it->second);  // re-insert moves to probation MRU
        const int n = (it != index_.end()) ? it->second : alloc(k);
        push_back(kProbation, n);
    }

    void touch(int64_t k) {
        auto it = index_.find(k);
        if (it == index_.end()) return;
        const int n = it->second;
        if (nodes_[n].seg == kProtected) {
            unlink(n);
            push_back(kProtected, n);
            return;
        }
        unlink(n);
        if (has_cap_) {
            const int64_t cap = std::max<int64_t>(1, (int64_t)((double)cap_ * ratio_));
            if (size_[kProtected] >= cap && size_[kProtected] > 0) {
                const int d = head_[kProtected];
                unlink(d);
                push_back(kProbation, d);
            }
        }
        push_back(kProtected, n);
    }

    bool pop_lru(int64_t* out) {
        for (int s : {kProbation, kProtected}) {
            if (head_[s] >= 0) {
                const int n = head_[s];
                *out = nodes_[n].key;
                erase_node(n);
                return true;
            }
        }
        return false;
    }

    bool pop_lru_excluding(const std::unordered_set<int64_t>& ex, int64_t* out) {
        for (int s : {kProbation, kProtected}) {
            for (int n = head_[s]; n >= 0; n = nodes_[n].next) {
                if (!ex.count(nodes_[n].key)) {
                    *out = nodes_[n].key;
                    erase_node(n);
                    return true;
                }
            }
        }
        return pop_lru(out);
    }

    void discard(int64_t k) {
        auto it = index_.find(k);
        if (it == index_.end()) return;
        erase_node(it->second);
    }

   private:
    static constexpr int kProbation = 0, kProtected = 1;
    struct Node {
        int64_t key;
        int prev, next, seg;
    };

    int alloc(int64_t k) {
        int n;
        if (!free_.empty()) {
            n = free_.back();
            free_.pop_back();
        } else {
            n = (int)nodes_.size();
            nodes_.push_back({});
        }
        nodes_[n] = {k, -1, -1, -1};
        index_[k] = n;
        return n;
    }
    void erase_node(int n) {
        unlink(n);
        index_.erase(nodes_[n].key);
        free_.push_back(n);
    }
    void unlink(int n) {
        Node& x = nodes_[n];
        if (x.seg < 0) return;
        if (x.prev >= 0) nodes_[x.prev].next = x.next; else head_[x.seg] = x.next;
        if (x.next >= 0) nodes_[x.next].prev = x.prev; else tail_[x.seg] = x.prev;
        size_[x.seg]--;
        x.prev = x.next = -1;
        x.seg = -1;
    }
    void push_back(int s, int n) {
        Node& x = nodes_[n];
        x.seg = s;
        x.prev = tail_[s];
        x.next = -1;
        if (tail_[s] >= 0) nodes_[tail_[s]].next = n; else head_[s] = n;
        tail_[s] = n;
        size_[s]++;
    }

    double ratio_;
    bool has_cap_ = false;
    int64_t cap_ = 0;
    std::vector<Node> nodes_;
    std::vector<int> free_;
    std::unordered_map<int64_t, int> index_;
    int head_[2], tail_[2];
    int64_t size_[2];
};

}  // namespace nvmoe

struct nvmoe_slru {
    nvmoe::SegmentedLru impl;
    explicit nvmoe_slru(double r) : impl(r) {}
};

extern "C" {

nvmoe_slru* nvmoe_slru_create(double protected_ratio) {
    if (!(protected_ratio >= 0.0) || !std::isfinite(protected_ratio)) return nullptr;
    return new (std::nothrow) nvmoe_slru(protected_ratio);
}
void nvmoe_slru_destroy(nvmoe_slru* lru) { delete lru; }
void nvmoe_slru_set_capacity_hint(nvmoe_slru* lru, int64_t c) {
    if (lru) lru->impl.set_capacity_hint(c);
}
void nvmoe_slru_insert_new(nvmoe_slru* lru, int64_t k) {
    if (lru) lru->impl.insert_new(k);
}
void nvmoe_slru_touch(nvmoe_slru* lru, int64_t k) {
    if (lru) lru->impl.touch(k);
}
int nvmoe_slru_contains(const nvmoe_slru* lru, int64_t k) {
    return lru && lru->impl.contains(k) ? 1 : 0;
}
int64_t nvmoe_slru_size(const nvmoe_slru* lru) { return lru ? lru->impl.size() : 0; }
int nvmoe_slru_pop_lru(nvmoe_slru* lru, int64_t* out) {
    if (!lru || !out) return NVMOE_ERR_INVALID_ARG;
    return lru->impl.pop_lru(out) ? NVMOE_OK : -1;
}
int nvmoe_slru_pop_lru_excluding(nvmoe_slru* lru, const int64_t* protect, int n, int64_t* out) {
    if (!lru || !out || n < 0 || (n > 0 && !protect)) return NVMOE_ERR_INVALID_ARG;
    std::unordered_set<int64_t> ex(protect, protect + n);
    return lru->impl.pop_lru_excluding(ex, out) ? NVMOE_OK : -1;
}
void nvmoe_slru_discard(nvmoe_slru* lru, int64_t k) {
    if (lru) lru->impl.discard(k);
}

}  // extern "C"

// ---------------------------------------------------------------- the bounded pinned host tier
// One layer's host tier of the llama.cpp engine (scripts/moe_cache_probe.cpp:636-752): a pool
// of host_slots pinned expert slots in front of the backing store, placed by the segmented LRU
// above.  nvmoe_host_tier_resolve is the host part of one eval_cb step, after the GPU remap.
struct nvmoe_host_tier {
    explicit nvmoe_host_tier(int32_t e, int32_t hs, double r)
        : n_expert(e), host_slots(hs), slot_of((size_t)e, -1), id_in((size_t)hs, -1), lru(r) {
        lru.set_capacity_hint(hs);
    }
    int32_t n_expert, host_slots, next_free = 0;
    std::vector<int32_t> slot_of;  // host slot of expert e, -1: not in the host tier
    std::vector<int32_t> id_in;    // expert in host slot h, -1: free
    nvmoe::SegmentedLru lru;
    std::unordered_set<int64_t> active;  // the step's distinct ids (reused)
    int64_t host_hits = 0, host_misses = 0;  // misses served by a host slot / loaded
};

extern "C" {

nvmoe_host_tier* nvmoe_host_tier_create(int32_t n_expert, int32_t host_slots,
                                        double protected_ratio) {
    if (n_expert <= 0 || host_slots <= 0 || !(protected_ratio >= 0.0) ||
        !std::isfinite(protected_ratio))
        return nullptr;
    return new nvmoe_host_tier(n_expert, host_slots, protected_ratio);
}

void nvmoe_host_tier_destroy(nvmoe_host_tier* t) { delete t; }

int nvmoe_host_tier_resolve(nvmoe_host_tier* t, const int32_t* unique_ids,
                            const uint8_t* unique_hit, int n_unique, const int32_t* miss_ids,
                            int n_miss, int32_t* host_slot_out, uint8_t* load_out) {
    if (!t || n_unique < 0 || n_miss < 0 || (n_unique > 0 && (!unique_ids || !unique_hit)) ||
        (n_miss > 0 && (!miss_ids || !host_slot_out || !load_out)))
        return NVMOE_ERR_INVALID_ARG;
    for (int i = 0; i < n_unique; ++i)
        if (unique_ids[i] < 0 || unique_ids[i] >= t->n_expert) return NVMOE_ERR_BAD_EXPERT_ID;
    for (int m = 0; m < n_miss; ++m)
        if (miss_ids[m] < 0 || miss_ids[m] >= t->n_expert) return NVMOE_ERR_BAD_EXPERT_ID;
    t->active.clear();
    for (int i = 0; i < n_unique; ++i) t->active.insert(unique_ids[i]);
    // GPU hits that are also in the host tier refresh it (moe_cache_probe.cpp:659-674)
    for (int i = 0; i < n_unique; ++i)
        if (unique_hit[i] && t->slot_of[(size_t)unique_ids[i]] != -1) t->lru.touch(unique_ids[i]);
    for (int m = 0; m < n_miss; ++m) {
        const int32_t r = miss_ids[m];
        const int32_t hs = t->slot_of[(size_t)r];
        if (hs != -1) {  // host hit: copy from its slot
            t->lru.touch(r);
            host_slot_out[m] = hs;
            load_out[m] = 0;
            ++t->host_hits;
            continue;
        }
        int32_t ns;
        if (t->next_free < t->host_slots) {
            ns = t->next_free++;
        } else {  // the least recent key not used by this step (probation first)
            int64_t victim = -1;
            if (!t->lru.pop_lru_excluding(t->active, &victim) && !t->lru.pop_lru(&victim))
                return NVMOE_ERR_CACHE_OVERFLOW;
            ns = t->slot_of[(size_t)victim];
            t->slot_of[(size_t)victim] = -1;
            t->id_in[(size_t)ns] = -1;
        }
        t->id_in[(size_t)ns] = r;
        t->slot_of[(size_t)r] = ns;
        t->lru.insert_new(r);
        host_slot_out[m] = ns;
        load_out[m] = 1;  // the caller fills host slot ns from the backing store
        ++t->host_misses;
    }
    return NVMOE_OK;
}

int nvmoe_host_tier_tables(const nvmoe_host_tier* t, int32_t* host_slot_of_id,
                           int32_t* id_in_host_slot) {
    if (!t) return NVMOE_ERR_INVALID_ARG;
    if (host_slot_of_id)
        std::copy(t->slot_of.begin(), t->slot_of.end(), host_slot_of_id);
    if (id_in_host_slot)
        std::copy(t->id_in.begin(), t->id_in.end(), id_in_host_slot);
    return NVMOE_OK;
}

int nvmoe_host_tier_stats(const nvmoe_host_tier* t, int64_t* host_hits, int64_t* host_misses) {
    if (!t) return NVMOE_ERR_INVALID_ARG;
    if (host_hits) *host_hits = t->host_hits;
    if (host_misses) *host_misses = t->host_misses;
    return NVMOE_OK;
}

}  // extern "C"
