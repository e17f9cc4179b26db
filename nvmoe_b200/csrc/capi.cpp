// Library-wide C ABI helpers: version string and the per-thread last-error text.
#include <cuda_runtime.h>

#include <cstdio>
#include <cstring>

#include "../../include/nvmoe_b200.h"

namespace nvmoe {

static thread_local char t_last_error[512] = "";

void set_last_error(const char* what, cudaError_t err) {
    std::snprintf(t_last_error, sizeof(t_last_error), "%s: %s (%s)", what ? what : "?",
                  cudaGetErrorName(err), cudaGetErrorString(err));
}

int cuda_status(const char* what, cudaError_t err) {
    if (err == cudaSuccess) return NVMOE_OK;
    set_last_error(what, err);
    return NVMOE_ERR_CUDA;
}

}  // namespace nvmoe

extern "C" const char* nvmoe_last_error(void) { return nvmoe::t_last_error; }

extern "C" const char* nvmoe_version(void) { return "nvmoe_b200 0.1.0 sm_100a"; }
