// C shim over the REFERENCE's own SegmentedHostLru (scripts/segmented_host_lru.hpp), compiled
// from the reference tree by oracle/Makefile into oracle/_ref/ (test infrastructure only).
// This file is ours; the header it includes is the reference's, used unmodified.
#include <cstdint>
#include <unordered_set>

#include "segmented_host_lru.hpp"

extern "C" {
void* ref_slru_create(double ratio) { return new SegmentedHostLru<int64_t>(ratio); }
void ref_slru_destroy(void* p) { delete static_cast<SegmentedHostLru<int64_t>*>(p); }
void ref_slru_set_capacity_hint(void* p, int64_t c) {
    static_cast<SegmentedHostLru<int64_t>*>(p)->set_capacity_hint(c);
}
void ref_slru_insert_new(void* p, int64_t k) { static_cast<SegmentedHostLru<int64_t>*>(p)->insert_new(k); }
void ref_slru_touch(void* p, int64_t k) { static_cast<SegmentedHostLru<int64_t>*>(p)->touch(k); }
int ref_slru_contains(void* p, int64_t k) { return static_cast<SegmentedHostLru<int64_t>*>(p)->contains(k); }
int64_t ref_slru_size(void* p) { return (int64_t) static_cast<SegmentedHostLru<int64_t>*>(p)->size(); }
int64_t ref_slru_pop_lru(void* p) { return static_cast<SegmentedHostLru<int64_t>*>(p)->pop_lru(); }
int64_t ref_slru_pop_lru_excluding(void* p, const int64_t* prot, int n) {
    std::unordered_set<int64_t> ex(prot, prot + n);
    return static_cast<SegmentedHostLru<int64_t>*>(p)->pop_lru_matching(
        [&](int64_t k) { return ex.count(k) == 0; });
}
void ref_slru_discard(void* p, int64_t k) { static_cast<SegmentedHostLru<int64_t>*>(p)->discard(k); }
}
