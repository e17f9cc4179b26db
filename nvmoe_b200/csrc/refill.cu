// R5 — refill of missed experts from the pinned host tier into their new device slots.
//
// Reference: gpu_fill_from_host_async (scripts/moe_cache_probe.cpp:377-404) issues one
// cudaMemcpyAsync per bank row on a high-priority h2d stream and joins the compute stream with
// an event (:988-993); the Python engine gathers all banks of all misses with one kernel over
// pinned host pointers (fast_index_copy_multi_jit, nvme_offload_cache.py:930-949, 1713-1720).
//
// nvmoe_refill_async  — copy engines: one cudaMemcpyAsync per (bank, run of consecutive slots)
//                       on the side stream, ordered after the compute stream's prior work (the
//                       evicted slot may still be read by an earlier FFN) and joined back.
// nvmoe_refill_gather — SM kernel for graph capture: reads the miss list written by the remap
//                       kernel and the host-tier slot of each miss from device memory, and copies
//                       from mapped pinned host memory with 16-byte loads (no host round trip).
#include "common.cuh"

#include <vector>

namespace nvmoe {
namespace {

constexpr int kMaxBanks = 8;
constexpr int64_t kPiece = 32 * 1024;

struct GatherParams {
    nvmoe_refill_bank banks[kMaxBanks];
    uint8_t vec16[kMaxBanks];  // bank rows, strides and bases all 16-byte aligned
    uint8_t vec4[kMaxBanks];   // ... 4-byte aligned
    int n_banks;
    int64_t max_pieces;  // pieces per (miss, bank) for the largest bank
    const int32_t* counts;
    int32_t* counts_rw;
    const int32_t* miss_ids;
    const int32_t* miss_slots;
    const int32_t* host_slot_of_id;
    int32_t n_gpu_slots;
};

__global__ void __launch_bounds__(256) refill_gather_kernel(GatherParams P) {
    grid_dep_wait();
    const int n_miss = P.counts[1];
    const int64_t jobs = (int64_t)n_miss * P.n_banks * P.max_pieces;
    for (int64_t job = blockIdx.x; job < jobs; job += gridDim.x) {
        const int64_t piece = job % P.max_pieces;
        const int64_t mb = job / P.max_pieces;
        const int b = (int)(mb % P.n_banks);
        const int m = (int)(mb / P.n_banks);
        const nvmoe_refill_bank& B = P.banks[b];
        const int64_t beg = piece * kPiece;
        if (beg >= B.row_bytes) continue;
        const int64_t end = min(B.row_bytes, beg + kPiece);
        const int gs = P.miss_slots[m];
        const int hs = P.host_slot_of_id[P.miss_ids[m]];
        if (hs < 0 || gs < 0 || gs >= P.n_gpu_slots) {
            if (threadIdx.x == 0) atomicExch(P.counts_rw + 2, NVMOE_ERR_HOST_LOAD);
            continue;
        }
        const char* src = static_cast<const char*>(B.src) + (int64_t)hs * B.src_slot_stride + beg;
        char* dst = static_cast<char*>(B.dst) + (int64_t)gs * B.dst_slot_stride + beg;
        const int64_t len = end - beg;
        if (P.vec16[b]) {  // 16-byte aligned bank: vector copy
            const int64_t n16 = len >> 4;
            for (int64_t i = threadIdx.x; i < n16; i += blockDim.x)
                reinterpret_cast<uint4*>(dst)[i] = reinterpret_cast<const uint4*>(src)[i];
        } else if (P.vec4[b]) {  // e.g. the fp32 global-scale bank (4 bytes per slot)
            for (int64_t i = threadIdx.x; i < (len >> 2); i += blockDim.x)
                reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
        } else {
            for (int64_t i = threadIdx.x; i < len; i += blockDim.x) dst[i] = src[i];
        }
    }
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_refill_async(const nvmoe_refill_bank* banks, int n_banks,
                                  const int32_t* gpu_slots, const int32_t* host_slots, int n,
                                  int32_t n_gpu_slots, int32_t n_host_slots,
                                  nvmoe_stream_t copy_stream, nvmoe_stream_t compute_stream,
                                  nvmoe_event_t done) {
    using namespace nvmoe;
    if (n < 0 || n_banks < 0 || (n > 0 && (!gpu_slots || !host_slots)) || (n_banks > 0 && !banks))
        return NVMOE_ERR_INVALID_ARG;
    for (int i = 0; i < n; ++i)
        if (gpu_slots[i] < 0 || gpu_slots[i] >= n_gpu_slots || host_slots[i] < 0 ||
            host_slots[i] >= n_host_slots)
            return NVMOE_ERR_INVALID_ARG;
    for (int b = 0; b < n_banks; ++b)
        if (!banks[b].dst || !banks[b].src || banks[b].row_bytes < 0) return NVMOE_ERR_INVALID_ARG;
    cudaStream_t cs = (cudaStream_t)copy_stream;
    cudaStream_t ks = (cudaStream_t)compute_stream;
    cudaEvent_t ev = (cudaEvent_t)done;
    if (n == 0) return NVMOE_OK;
    // the evicted slots may still be read by FFN work queued earlier on the compute stream
    // (a null compute stream is the default stream, a stream like any other here)
    if (ev && ks != cs) {
        NVMOE_CUDA_TRY(cudaEventRecord(ev, ks));
        NVMOE_CUDA_TRY(cudaStreamWaitEvent(cs, ev, 0));
    }
    for (int b = 0; b < n_banks; ++b) {
        const nvmoe_refill_bank& B = banks[b];
        if (B.row_bytes == 0) continue;
        const bool dense = B.dst_slot_stride == B.row_bytes && B.src_slot_stride == B.row_bytes;
        int i = 0;
        while (i < n) {
            int j = i + 1;
            if (dense)
                while (j < n && gpu_slots[j] == gpu_slots[j - 1] + 1 &&
                       host_slots[j] == host_slots[j - 1] + 1)
                    ++j;
            char* dst = static_cast<char*>(B.dst) + (int64_t)gpu_slots[i] * B.dst_slot_stride;
            const char* src =
                static_cast<const char*>(B.src) + (int64_t)host_slots[i] * B.src_slot_stride;
            NVMOE_CUDA_TRY(cudaMemcpyAsync(dst, src, (size_t)B.row_bytes * (j - i),
                                           cudaMemcpyHostToDevice, cs));
            i = j;
        }
    }
    if (ev) {
        NVMOE_CUDA_TRY(cudaEventRecord(ev, cs));
        if (ks != cs) NVMOE_CUDA_TRY(cudaStreamWaitEvent(ks, ev, 0));
    }
    return NVMOE_OK;
}

extern "C" int nvmoe_refill_gather(const nvmoe_refill_bank* banks, int n_banks,
                                   const nvmoe_miss_list* misses, const int32_t* host_slot_of_id,
                                   int32_t n_gpu_slots, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!banks || n_banks <= 0 || n_banks > kMaxBanks || !misses || !host_slot_of_id ||
        !misses->counts || !misses->miss_ids || !misses->miss_slots || n_gpu_slots <= 0)
        return NVMOE_ERR_INVALID_ARG;
    GatherParams P;
    P.n_banks = n_banks;
    int64_t maxp = 1;
    for (int b = 0; b < n_banks; ++b) {
        const nvmoe_refill_bank& B = banks[b];
        if (!B.dst || !B.src || B.row_bytes < 0) return NVMOE_ERR_INVALID_ARG;
        const uint64_t bits = (uint64_t)B.row_bytes | (uint64_t)B.dst_slot_stride |
                              (uint64_t)B.src_slot_stride | reinterpret_cast<uintptr_t>(B.dst) |
                              reinterpret_cast<uintptr_t>(B.src);
        P.banks[b] = B;
        // pieces start at multiples of kPiece (a multiple of 16), so base alignment is kept
        P.vec16[b] = (bits & 15) == 0;
        P.vec4[b] = (bits & 3) == 0;
        const int64_t pcs = (B.row_bytes + kPiece - 1) / kPiece;
        if (pcs > maxp) maxp = pcs;
    }
    P.max_pieces = maxp;
    P.counts = misses->counts;
    P.counts_rw = misses->counts;
    P.miss_ids = misses->miss_ids;
    P.miss_slots = misses->miss_slots;
    P.host_slot_of_id = host_slot_of_id;
    P.n_gpu_slots = n_gpu_slots;
    cudaError_t e = launch_pdl(refill_gather_kernel, dim3(kNumSMs * 2), dim3(256), 0,
                               (cudaStream_t)stream, true, P);
    return cuda_status("refill_gather launch", e);
}
