/*
 * CPU oracle (test infrastructure only): serial restatement of the llama.cpp engine's
 * expert-cache callback, scripts/moe_cache_probe.cpp:eval_cb, GPU tier + host tier.
 *
 *   :627-634  distinct ids, first-occurrence order (linear std::find scan)
 *   :636-674  ++current_step; GPU hits: slot_last_used[slot] = step, host-resident hits
 *             touch the host LRU; GPU misses collected in order
 *   :676-722  per miss: scan [start, cache_size) (start = gpu_pinned_k in decode): first empty
 *             slot wins immediately, else the smallest slot_last_used (strict <) among slots
 *             whose occupant is not a distinct id of this call; none -> rescan [0, cache_size);
 *             none again -> overflow (reference: abort); stamp, evict, install
 *   :724-752  host tier: host-resident miss -> touch + H2D from that host slot; otherwise a
 *             host slot from host_next_free, else SegmentedHostLru::pop_lru_matching(not in the
 *             active set) (scripts/segmented_host_lru.hpp:130-141), insert_new -> load task
 *   :955-970  rewrite ids -> slots
 *
 * The host LRU is restated here as well (nvme_offload_cache.py:333-409 /
 * segmented_host_lru.hpp:85-160), keyed by expert id.
 */
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

/* ------------------------------------------------------------------ SLRU (two linked lists) */
typedef struct {
    int n_keys;
    int32_t *prev, *next; /* per key */
    int8_t* seg;          /* -1 absent, 0 probation, 1 protected */
    int32_t head[2], tail[2];
    int64_t size[2];
    double ratio;
    int has_cap;
    int64_t cap;
} orc_slru;

static void slru_init(orc_slru* l, int n_keys, double ratio) {
    l->n_keys = n_keys;
    l->prev = (int32_t*)malloc(sizeof(int32_t) * n_keys);
    l->next = (int32_t*)malloc(sizeof(int32_t) * n_keys);
    l->seg = (int8_t*)malloc(n_keys);
    for (int i = 0; i < n_keys; ++i) l->prev[i] = l->next[i] = -1, l->seg[i] = -1;
    l->head[0] = l->head[1] = l->tail[0] = l->tail[1] = -1;
    l->size[0] = l->size[1] = 0;
    l->ratio = ratio;
    l->has_cap = 0;
    l->cap = 0;
}
static void slru_free(orc_slru* l) {
    free(l->prev);
    free(l->next);
    free(l->seg);
}
static void slru_unlink(orc_slru* l, int k) {
    int s = l->seg[k];
    if (s < 0) return;
    if (l->prev[k] >= 0) l->next[l->prev[k]] = l->next[k]; else l->head[s] = l->next[k];
    if (l->next[k] >= 0) l->prev[l->next[k]] = l->prev[k]; else l->tail[s] = l->prev[k];
    l->prev[k] = l->next[k] = -1;
    l->seg[k] = -1;
    l->size[s]--;
}
static void slru_push_back(orc_slru* l, int s, int k) {
    l->seg[k] = (int8_t)s;
    l->prev[k] = l->tail[s];
    l->next[k] = -1;
    if (l->tail[s] >= 0) l->next[l->tail[s]] = k; else l->head[s] = k;
    l->tail[s] = k;
    l->size[s]++;
}
static void slru_set_capacity_hint(orc_slru* l, int64_t c) {
    if (!l->has_cap) l->has_cap = 1, l->cap = c;
}
static void slru_insert_new(orc_slru* l, int k) {
    slru_unlink(l, k);
    slru_push_back(l, 0, k);
}
static void slru_touch(orc_slru* l, int k) {
    if (l->seg[k] == 1) {
        slru_unlink(l, k);
        slru_push_back(l, 1, k);
        return;
    }
    if (l->seg[k] == 0) {
        slru_unlink(l, k);
        if (l->has_cap) {
            int64_t cap = (int64_t)((double)l->cap * l->ratio);
            if (cap < 1) cap = 1;
            if (l->size[1] >= cap && l->size[1] > 0) {
                int d = l->head[1];
                slru_unlink(l, d);
                slru_push_back(l, 0, d);
            }
        }
        slru_push_back(l, 1, k);
    }
}
static int slru_pop_lru(orc_slru* l) {
    for (int s = 0; s < 2; ++s)
        if (l->head[s] >= 0) {
            int k = l->head[s];
            slru_unlink(l, k);
            return k;
        }
    return -1;
}
/* excluded[k] != 0: key protected from eviction */
static int slru_pop_lru_matching(orc_slru* l, const uint8_t* excluded) {
    for (int s = 0; s < 2; ++s)
        for (int k = l->head[s]; k >= 0; k = l->next[k])
            if (!excluded[k]) {
                slru_unlink(l, k);
                return k;
            }
    return slru_pop_lru(l);
}

/* ------------------------------------------------------------------ exported SLRU (keys < n) */
void* orc_slru_create(int n_keys, double ratio) {
    orc_slru* l = (orc_slru*)malloc(sizeof(orc_slru));
    slru_init(l, n_keys, ratio);
    return l;
}
void orc_slru_destroy(void* p) {
    slru_free((orc_slru*)p);
    free(p);
}
void orc_slru_set_capacity_hint(void* p, int64_t c) { slru_set_capacity_hint((orc_slru*)p, c); }
void orc_slru_insert_new(void* p, int k) { slru_insert_new((orc_slru*)p, k); }
void orc_slru_touch(void* p, int k) { slru_touch((orc_slru*)p, k); }
int orc_slru_contains(void* p, int k) { return ((orc_slru*)p)->seg[k] >= 0; }
int64_t orc_slru_size(void* p) { return ((orc_slru*)p)->size[0] + ((orc_slru*)p)->size[1]; }
int orc_slru_pop_lru(void* p) { return slru_pop_lru((orc_slru*)p); }
int orc_slru_pop_lru_excluding(void* p, const int32_t* prot, int n) {
    orc_slru* l = (orc_slru*)p;
    uint8_t* ex = (uint8_t*)calloc(l->n_keys, 1);
    for (int i = 0; i < n; ++i)
        if (prot[i] >= 0 && prot[i] < l->n_keys) ex[prot[i]] = 1;
    int k = slru_pop_lru_matching(l, ex);
    free(ex);
    return k;
}
void orc_slru_discard(void* p, int k) { slru_unlink((orc_slru*)p, k); }

/* ------------------------------------------------------------------ layer cache */
typedef struct {
    int n_expert, cache_size, pinned_k, host_cache_size;
    int32_t* slot_of_real;   /* [n_expert] */
    int32_t* real_in_slot;   /* [cache_size] */
    uint32_t* slot_last_used;/* [cache_size] */
    uint32_t current_step;
    int32_t* host_slot_of_real; /* [n_expert] */
    int32_t* host_real_in_slot; /* [host_cache_size] */
    int32_t host_next_free;
    orc_slru lru;
} orc_layer;

void* orc_layer_create(int n_expert, int cache_size, int pinned_k, int host_cache_size,
                       double protected_ratio) {
    orc_layer* L = (orc_layer*)calloc(1, sizeof(orc_layer));
    L->n_expert = n_expert;
    L->cache_size = cache_size;
    L->pinned_k = pinned_k;
    L->host_cache_size = host_cache_size;
    L->slot_of_real = (int32_t*)malloc(4 * (size_t)n_expert);
    L->real_in_slot = (int32_t*)malloc(4 * (size_t)cache_size);
    L->slot_last_used = (uint32_t*)calloc((size_t)cache_size, 4);
    L->host_slot_of_real = (int32_t*)malloc(4 * (size_t)n_expert);
    L->host_real_in_slot = (int32_t*)malloc(4 * (size_t)(host_cache_size > 0 ? host_cache_size : 1));
    for (int i = 0; i < n_expert; ++i) L->slot_of_real[i] = -1, L->host_slot_of_real[i] = -1;
    for (int i = 0; i < cache_size; ++i) L->real_in_slot[i] = -1;
    for (int i = 0; i < host_cache_size; ++i) L->host_real_in_slot[i] = -1;
    slru_init(&L->lru, n_expert, protected_ratio);
    slru_set_capacity_hint(&L->lru, host_cache_size);
    return L;
}

void orc_layer_destroy(void* p) {
    orc_layer* L = (orc_layer*)p;
    free(L->slot_of_real);
    free(L->real_in_slot);
    free(L->slot_last_used);
    free(L->host_slot_of_real);
    free(L->host_real_in_slot);
    slru_free(&L->lru);
    free(L);
}

/* Raw table access for tests (copy out / in). */
void orc_layer_tables(void* p, int32_t* slot_of_real, int32_t* real_in_slot,
                      uint32_t* slot_last_used, uint32_t* step) {
    orc_layer* L = (orc_layer*)p;
    if (slot_of_real) memcpy(slot_of_real, L->slot_of_real, 4 * (size_t)L->n_expert);
    if (real_in_slot) memcpy(real_in_slot, L->real_in_slot, 4 * (size_t)L->cache_size);
    if (slot_last_used) memcpy(slot_last_used, L->slot_last_used, 4 * (size_t)L->cache_size);
    if (step) *step = L->current_step;
}
void orc_layer_set_tables(void* p, const int32_t* slot_of_real, const int32_t* real_in_slot,
                          const uint32_t* slot_last_used, uint32_t step) {
    orc_layer* L = (orc_layer*)p;
    memcpy(L->slot_of_real, slot_of_real, 4 * (size_t)L->n_expert);
    memcpy(L->real_in_slot, real_in_slot, 4 * (size_t)L->cache_size);
    memcpy(L->slot_last_used, slot_last_used, 4 * (size_t)L->cache_size);
    L->current_step = step;
}
void orc_layer_host_tables(void* p, int32_t* host_slot_of_real, int32_t* host_real_in_slot) {
    orc_layer* L = (orc_layer*)p;
    if (host_slot_of_real) memcpy(host_slot_of_real, L->host_slot_of_real, 4 * (size_t)L->n_expert);
    if (host_real_in_slot && L->host_cache_size > 0)
        memcpy(host_real_in_slot, L->host_real_in_slot, 4 * (size_t)L->host_cache_size);
}

static int find_int(const int32_t* a, int n, int32_t v) {
    for (int i = 0; i < n; ++i)
        if (a[i] == v) return i;
    return -1;
}

/*
 * One callback.  ids: n = n_tok * top_k expert ids (contiguous).  Outputs (capacity n):
 *   out_slots[n], unique_ids[*n_unique], unique_hit[*n_unique], miss_ids / miss_slots /
 *   evicted[*n_miss]; host tier (when with_host != 0): h2d_gpu[*n_h2d] / h2d_host[*n_h2d] for
 *   host hits, load_ids / load_gpu / load_host[*n_load] for host misses.
 * Returns 0, -2 (bad id: reference logs [BUG] after indexing out of bounds; here nothing is
 * modified), -3 (no victim: reference aborts) or -4 (host tier without any slot).
 */
int orc_layer_eval(void* p, const int32_t* ids, int n, int is_decode, int with_host,
                   int32_t* out_slots, int32_t* unique_ids, uint8_t* unique_hit, int32_t* n_unique,
                   int32_t* miss_ids, int32_t* miss_slots, int32_t* evicted, int32_t* n_miss,
                   int32_t* h2d_gpu, int32_t* h2d_host, int32_t* n_h2d, int32_t* load_ids,
                   int32_t* load_gpu, int32_t* load_host, int32_t* n_load) {
    orc_layer* L = (orc_layer*)p;
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= L->n_expert) return -2;
    int nu = 0;
    for (int i = 0; i < n; ++i)
        if (find_int(unique_ids, nu, ids[i]) < 0) unique_ids[nu++] = ids[i];
    *n_unique = nu;
    /* A victim exists for every miss iff the distinct ids fit in the pool (nu <= cache_size);
     * the reference aborts when they do not (moe_cache_probe.cpp:709-712).  Detect it before
     * any state changes, like the device kernel. */
    if (nu > L->cache_size) return -3;
    uint8_t* active = (uint8_t*)calloc((size_t)L->n_expert, 1);
    for (int i = 0; i < nu; ++i) active[unique_ids[i]] = 1;

    L->current_step++;
    int nm = 0;
    for (int i = 0; i < nu; ++i) {
        int r = unique_ids[i];
        int s = L->slot_of_real[r];
        if (s != -1) {
            unique_hit[i] = 1;
            L->slot_last_used[s] = L->current_step;
            if (with_host && L->host_slot_of_real[r] != -1) slru_touch(&L->lru, r);
        } else {
            unique_hit[i] = 0;
            miss_ids[nm++] = r;
        }
    }
    *n_miss = nm;
    int nh = 0, nl = 0;
    for (int m = 0; m < nm; ++m) {
        int r = miss_ids[m];
        int chosen = -1;
        uint32_t oldest = UINT32_MAX;
        int start = (is_decode && L->pinned_k > 0) ? L->pinned_k : 0;
        for (int s = start; s < L->cache_size; ++s) {
            int occ = L->real_in_slot[s];
            if (occ == -1) {
                chosen = s;
                break;
            }
            if (!active[occ] && L->slot_last_used[s] < oldest) {
                oldest = L->slot_last_used[s];
                chosen = s;
            }
        }
        if (chosen == -1) {
            for (int s = 0; s < L->cache_size; ++s) {
                int occ = L->real_in_slot[s];
                if (occ == -1) {
                    chosen = s;
                    break;
                }
                if (!active[occ] && L->slot_last_used[s] < oldest) {
                    oldest = L->slot_last_used[s];
                    chosen = s;
                }
            }
        }
        if (chosen == -1) {
            free(active);
            return -3;
        }
        L->slot_last_used[chosen] = L->current_step;
        int ev = L->real_in_slot[chosen];
        if (ev != -1) L->slot_of_real[ev] = -1;
        L->real_in_slot[chosen] = r;
        L->slot_of_real[r] = chosen;
        miss_slots[m] = chosen;
        evicted[m] = ev;
        if (with_host) {
            int hs = L->host_slot_of_real[r];
            if (hs != -1) {
                slru_touch(&L->lru, r);
                h2d_gpu[nh] = chosen;
                h2d_host[nh] = hs;
                nh++;
            } else {
                int ns;
                if (L->host_next_free < L->host_cache_size) {
                    ns = L->host_next_free++;
                } else {
                    int victim = slru_pop_lru_matching(&L->lru, active);
                    if (victim < 0) {  /* empty host LRU: the reference would read garbage */
                        free(active);
                        return -4;
                    }
                    ns = L->host_slot_of_real[victim];
                    L->host_slot_of_real[victim] = -1;
                    L->host_real_in_slot[ns] = -1;
                }
                L->host_real_in_slot[ns] = r;
                L->host_slot_of_real[r] = ns;
                slru_insert_new(&L->lru, r);
                load_ids[nl] = r;
                load_gpu[nl] = chosen;
                load_host[nl] = ns;
                nl++;
            }
        }
    }
    if (n_h2d) *n_h2d = nh;
    if (n_load) *n_load = nl;
    for (int i = 0; i < n; ++i) out_slots[i] = L->slot_of_real[ids[i]];
    free(active);
    return 0;
}
