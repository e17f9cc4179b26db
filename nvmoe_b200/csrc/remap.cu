// R2 / R3 / R6 — expert-id -> slot remap with hit / miss lists, on the device.
//
// Reference: the GPU-tier half of eval_cb, scripts/moe_cache_probe.cpp:
//   :627-634  distinct ids in first-occurrence order
//   :636-674  hits refresh slot_last_used[slot] = current_step (after ++current_step)
//   :676-722  each miss, in order, takes the first empty slot in [start, cache_size), else the
//             slot with the smallest slot_last_used (strict <, so ties go to the lowest slot)
//             whose occupant is not among this call's distinct ids; start = gpu_pinned_k in
//             decode, 0 otherwise; with no candidate there, the same rule over [0, start)
//   :707-722  evict the old occupant, install the miss, stamp slot_last_used
//   :955-970  rewrite every id to its slot (ids are a strided view, row stride nb[1])
//
// Parallel formulation.  During one call the last-used stamps of non-active slots never
// change, and a slot taken by a miss becomes active.  The sequence of victims chosen by the
// serial scan is therefore the ascending order of the candidate key
//     (class, last_used, slot)   class 0: empty slot >= start   (last_used ignored)
//                                class 1: non-active slot >= start
//                                class 2: empty slot < start
//                                class 3: non-active slot < start
// and miss j (j-th miss in first-occurrence order) gets the j-th smallest key.  The kernel
// computes that with one bitonic sort of the slot keys in shared memory.
//
// One CTA does the whole call: distinct ids via atomicMin of the first position per id,
// ordered compaction with warp ballots + a block scan, then the sort.  Invalid ids or more
// distinct ids than slots leave the tables untouched and report an error status.
#include "remap_device.cuh"

namespace nvmoe {
namespace {

constexpr int kRemapThreads = 1024;

__global__ void __launch_bounds__(kRemapThreads, 1) remap_kernel(RemapParams P) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    remap_block(P, smem_raw);
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_remap(const nvmoe_slot_table* table, const int32_t* ids,
                           int64_t ids_row_stride_bytes, int top_k, int n_tok, int is_decode,
                           int32_t* out_slots, int64_t out_row_stride_bytes,
                           const nvmoe_miss_list* misses, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!table || !misses || !ids || !out_slots) return NVMOE_ERR_INVALID_ARG;
    const nvmoe_slot_table& t = *table;
    if (!t.slot_of_real || !t.real_in_slot || !t.slot_last_used || !t.current_step)
        return NVMOE_ERR_INVALID_ARG;
    if (t.n_expert <= 0 || t.n_expert > kMaxExpertsRemap || t.cache_size <= 0 ||
        t.cache_size > kMaxSlotsRemap || t.pinned_k < 0 || t.id_base < 0)
        return NVMOE_ERR_INVALID_ARG;
    if (top_k <= 0 || n_tok < 0) return NVMOE_ERR_INVALID_ARG;
    if (ids_row_stride_bytes < (int64_t)top_k * 4 || out_row_stride_bytes < (int64_t)top_k * 4 ||
        (ids_row_stride_bytes & 3) || (out_row_stride_bytes & 3))
        return NVMOE_ERR_INVALID_ARG;
    const int64_t n = (int64_t)n_tok * top_k;
    if (n > (1 << 24)) return NVMOE_ERR_INVALID_ARG;
    const nvmoe_miss_list& m = *misses;
    if (!m.unique_ids || !m.unique_slot || !m.unique_hit || !m.miss_ids || !m.miss_slots ||
        !m.evicted_ids || !m.counts)
        return NVMOE_ERR_INVALID_ARG;
    // lists hold at most min(n, n_expert) entries
    const int64_t need = n < t.n_expert ? n : t.n_expert;
    if (m.capacity < need) return NVMOE_ERR_INVALID_ARG;

    RemapParams P;
    P.t = t;
    P.ids = ids;
    P.ids_stride = ids_row_stride_bytes;
    P.out = out_slots;
    P.out_stride = out_row_stride_bytes;
    P.top_k = top_k;
    P.n_tok = n_tok;
    P.is_decode = is_decode;
    P.m = m;
    const size_t smem = remap_smem_bytes(t.n_expert, t.cache_size);
    if (smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
    if (smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(remap_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)smem));
    const int threads = n <= 256 && t.cache_size <= 512 ? 256 : kRemapThreads;
    remap_kernel<<<1, threads, smem, (cudaStream_t)stream>>>(P);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}
