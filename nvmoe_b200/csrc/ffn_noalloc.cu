// Allocation-free variant of the routed-expert FFN entry point (nvmoe_moe_ffn_noalloc).
//
// Some callers cannot allocate device memory at the moment they need the FFN: the llama.cpp
// eval callback, for example, runs on ggml's scheduler thread between graph nodes, where every
// device buffer belongs to ggml's allocator; a cudaMalloc there would synchronise the device in
// the middle of the graph and sit outside the framework's memory budget.  Processes that have
// handed all spare VRAM to the expert-slot pool are in the same position.  This entry point
// therefore takes no workspace: its scratch is one file-scope device array compiled into the
// library, and it calls no allocator at any point.
//
// Properties a caller must know:
//   - the scratch array (kNoAllocScratchBytes, 16 MiB) exists on every GPU that loads this part
//     of the library and stays allocated until the process exits;
//   - calls whose workspace requirement (nvmoe_moe_ffn_workspace_size) exceeds that size are
//     rejected with NVMOE_ERR_SCRATCH_LIMIT, before anything is launched;
//   - the first call on a device looks up the array's device address with
//     cudaGetSymbolAddress (once per device, with that device current); make that first call
//     before any stream capture.  The address is kept for the life of the process: it does
//     not survive cudaDeviceReset (or any other teardown of the device's primary context),
//     after which the array may sit elsewhere; a process that resets a device must not call
//     this entry point on it again;
//   - every call on a device shares the one array, which keeps the previous call's contents
//     (nothing in it has to start at zero: each call writes every scratch word before reading
//     it); calls that overlap on the GPU (different streams, or different host threads without
//     ordering) race on it and must be serialised by the caller.
#include "common.cuh"
#include "ffn_common.cuh"

#include <mutex>

namespace nvmoe {

int ffn_launch_prep(FfnParams& P, cudaStream_t st);

namespace {

constexpr size_t kNoAllocScratchBytes = 16u << 20;

static __device__ __align__(256) unsigned char g_ffn_scratch[kNoAllocScratchBytes];

std::mutex g_scratch_mu;
void* g_scratch_ptr[64];  // device address of g_ffn_scratch per device (null = not looked up)

int scratch_for_current_device(void** out) {
    int dev = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return NVMOE_ERR_UNSUPPORTED;
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        NVMOE_CUDA_TRY(cudaGetSymbolAddress(&p, g_ffn_scratch));
        if (!p) return NVMOE_ERR_CUDA;
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
    return NVMOE_OK;
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_moe_ffn_noalloc(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!args || !args->pool || args->n_tok < 0 || args->top_k <= 0) return NVMOE_ERR_INVALID_ARG;
    if (args->n_tok == 0) return NVMOE_OK;
    const nvmoe_expert_pool& pool = *args->pool;
    if (pool.hidden <= 0 || pool.inter <= 0 || pool.n_slots <= 0) return NVMOE_ERR_INVALID_ARG;
    const size_t need = ws_layout(args->n_tok, args->top_k, pool.hidden, pool.inter,
                                  pool.n_slots).total;
    if (need > kNoAllocScratchBytes) return NVMOE_ERR_SCRATCH_LIMIT;
    void* scratch = nullptr;
    const int rs = scratch_for_current_device(&scratch);
    if (rs != NVMOE_OK) return rs;
    nvmoe_ffn_args a = *args;
    a.workspace = scratch;
    a.workspace_bytes = kNoAllocScratchBytes;
    FfnParams P;
    const int rc = ffn_setup(&a, P);
    if (rc != NVMOE_OK) return rc;
    cudaStream_t st = (cudaStream_t)stream;
    const int r1 = ffn_launch_prep(P, st);
    if (r1 != NVMOE_OK) return r1;
    return ffn_launch_main(P, st);
}
