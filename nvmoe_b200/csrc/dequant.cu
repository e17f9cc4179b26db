// R8 — dequantisation of slot-pool weights to fp32 memory (bit-exact reference path).
//
// NVFP4 (FTW banks, scripts/convert_ftw_to_gguf.py:46-58 / nvme_offload_cache.py:824-835):
//   value = (e2m1(code) * e4m3(scale)) * global; codes packed two per byte, w[2b] in the low
//   nibble; one E4M3 scale per 16 consecutive values of a row.
// Q2_K (ggml block_q2_K, 84 bytes / 256 values): scales[16] (low nibble scale, high nibble min),
//   qs[64] (2-bit), fp16 d, fp16 dmin.  value = d*sc*q - dmin*m with fp32 roundings after each
//   product and after the subtraction (no FMA), value index e -> qs[32*(e/128) + e%32] >>
//   2*((e%128)/32).
// IQ2_XXS (ggml block_iq2_xxs, 66 bytes / 256 values): fp16 d, then per 32 values two u32:
//   four codebook indices (bytes) and (4 x 7-bit sign indices | 4-bit scale << 28).
//   db = d*(0.5+s)*0.25; value = db * grid[idx][i] * sign, sign bit i of
//   ksigns[j] = j | parity(j) << 7.
#include "common.cuh"

#include <mutex>

namespace nvmoe {

// IQ2_XXS codebook (256 entries x 8 magnitudes) in device global memory, per device.
__device__ uint8_t g_iq2xxs_grid[256 * 8];
static bool g_grid_ready[64];
static std::mutex g_grid_mu;

bool iq2xxs_grid_ready(int device) {
    std::lock_guard<std::mutex> lk(g_grid_mu);
    return device >= 0 && device < 64 && g_grid_ready[device];
}

const uint8_t* iq2xxs_grid_device_ptr() {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_iq2xxs_grid) != cudaSuccess) return nullptr;
    return static_cast<const uint8_t*>(p);
}

namespace {

__device__ __forceinline__ float e2m1_to_f32(uint32_t nib) {
    // exact E2M1 decode (s e1 e0 m); the negative-zero code 0x8 decodes to +0 like ggml's table
    const uint32_t mag = nib & 7u;
    const float v = (mag < 2u) ? 0.5f * (float)mag
                               : (float)(2u + (mag & 1u)) * exp2f((float)((mag >> 1) - 1u)) * 0.5f;
    return (nib & 8u) && mag ? -v : v;
}

__device__ __forceinline__ float e4m3_to_f32(uint8_t b) {
    const uint32_t s = b >> 7, e = (b >> 3) & 0xF, m = b & 7;
    float v;
    if (e == 0xF && m == 7) {
        v = __int_as_float(0x7fc00000);  // NaN (float8_e4m3fn)
    } else if (e == 0) {
        v = (float)m * 0.001953125f;  // m * 2^-9
    } else {
        v = (1.0f + (float)m * 0.125f) * exp2f((float)e - 7.0f);
    }
    return s ? -v : v;
}

__device__ __forceinline__ float half_bits_to_f32(uint16_t h) {
    return __half2float(__ushort_as_half(h));
}

__global__ void dequant_nvfp4_kernel(const uint8_t* __restrict__ codes,
                                     const uint8_t* __restrict__ scales,
                                     const float* __restrict__ global, int64_t n_rows,
                                     int64_t n_cols, float* __restrict__ out) {
    const int64_t half_cols = n_cols / 2;
    const int64_t total = n_rows * half_cols;
    const float g = global ? *global : 1.0f;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t r = i / half_cols, cb = i - r * half_cols;
        const uint8_t b = codes[i];
        const float sc = e4m3_to_f32(scales[r * (n_cols / 16) + (cb * 2) / 16]);
        const float v0 = __fmul_rn(__fmul_rn(e2m1_to_f32(b & 0xF), sc), g);
        const float v1 = __fmul_rn(__fmul_rn(e2m1_to_f32(b >> 4), sc), g);
        out[r * n_cols + cb * 2] = v0;
        out[r * n_cols + cb * 2 + 1] = v1;
    }
}

__global__ void dequant_q2k_kernel(const uint8_t* __restrict__ blocks, int64_t n_blocks,
                                   float* __restrict__ out) {
    const int64_t total = n_blocks * 256;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i >> 8;
        const int e = (int)(i & 255);
        const uint8_t* b = blocks + blk * 84;
        const uint8_t sc = b[e >> 4];
        const uint8_t q = (b[16 + 32 * (e >> 7) + (e & 31)] >> (2 * ((e & 127) >> 5))) & 3;
        const float d = half_bits_to_f32((uint16_t)(b[80] | (b[81] << 8)));
        const float dmin = half_bits_to_f32((uint16_t)(b[82] | (b[83] << 8)));
        const float dl = __fmul_rn(d, (float)(sc & 0xF));
        const float ml = __fmul_rn(dmin, (float)(sc >> 4));
        out[i] = __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
}

__global__ void dequant_iq2xxs_kernel(const uint8_t* __restrict__ blocks, int64_t n_blocks,
                                      float* __restrict__ out) {
    const int64_t total = n_blocks * 256;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t blk = i >> 8;
        const int e = (int)(i & 255);
        const uint8_t* b = blocks + blk * 66;
        const float d = half_bits_to_f32((uint16_t)(b[0] | (b[1] << 8)));
        const int g = e >> 5, l = (e >> 3) & 3, j = e & 7;
        const uint8_t* q = b + 2 + g * 8;
        const uint32_t aux1 = (uint32_t)q[4] | ((uint32_t)q[5] << 8) | ((uint32_t)q[6] << 16) |
                              ((uint32_t)q[7] << 24);
        const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux1 >> 28))), 0.25f);
        const uint32_t sidx = (aux1 >> (7 * l)) & 127u;
        const uint32_t signs = sidx | ((__popc(sidx) & 1u) << 7);
        const float mag = (float)g_iq2xxs_grid[q[l] * 8 + j];
        const float v = __fmul_rn(db, mag);
        out[i] = ((signs >> j) & 1u) ? -v : v;
    }
}

int grid_for(int64_t n) {
    int64_t g = (n + 255) / 256;
    if (g > 148 * 32) g = 148 * 32;
    return (int)(g < 1 ? 1 : g);
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_dequant_nvfp4(const uint8_t* codes, const uint8_t* scales,
                                   const float* global_scale, int64_t n_rows, int64_t n_cols,
                                   float* out, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!codes || !scales || !out || n_rows < 0 || n_cols < 0 || (n_cols % 16))
        return NVMOE_ERR_INVALID_ARG;
    if (n_rows == 0 || n_cols == 0) return NVMOE_OK;
    dequant_nvfp4_kernel<<<grid_for(n_rows * n_cols / 2), 256, 0, (cudaStream_t)stream>>>(
        codes, scales, global_scale, n_rows, n_cols, out);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}

extern "C" int nvmoe_dequant_q2_k(const void* blocks, int64_t n_blocks, float* out,
                                  nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!blocks || !out || n_blocks < 0) return NVMOE_ERR_INVALID_ARG;
    if (n_blocks == 0) return NVMOE_OK;
    dequant_q2k_kernel<<<grid_for(n_blocks * 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(blocks), n_blocks, out);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}

extern "C" int nvmoe_dequant_iq2_xxs(const void* blocks, int64_t n_blocks, float* out,
                                     nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!blocks || !out || n_blocks < 0) return NVMOE_ERR_INVALID_ARG;
    int dev = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    if (!iq2xxs_grid_ready(dev)) return NVMOE_ERR_NO_TABLES;
    if (n_blocks == 0) return NVMOE_OK;
    dequant_iq2xxs_kernel<<<grid_for(n_blocks * 256), 256, 0, (cudaStream_t)stream>>>(
        static_cast<const uint8_t*>(blocks), n_blocks, out);
    NVMOE_CUDA_TRY(cudaGetLastError());
    return NVMOE_OK;
}

extern "C" int nvmoe_set_iq2xxs_grid(const uint8_t* grid_256x8) {
    using namespace nvmoe;
    if (!grid_256x8) return NVMOE_ERR_INVALID_ARG;
    int dev = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return NVMOE_ERR_UNSUPPORTED;
    NVMOE_CUDA_TRY(cudaMemcpyToSymbol(g_iq2xxs_grid, grid_256x8, 256 * 8));
    NVMOE_CUDA_TRY(cudaDeviceSynchronize());
    std::lock_guard<std::mutex> lk(g_grid_mu);
    g_grid_ready[dev] = true;
    return NVMOE_OK;
}
