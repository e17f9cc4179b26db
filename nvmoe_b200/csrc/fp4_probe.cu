// Block-scaled FP4 tensor-core throughput of this GPU (nvmoe_probe_fp4_mma): the denominator the
// prefill's FP4 tensor roofline is measured against, since no FP4 peak is measured for the pool.
//
// One CTA per SM issues, from one thread, back-to-back tcgen05.mma kind::mxf4nvf4.block16 with
// exactly the prefill kernel's shape and operand layout (prefill_fp4.cu): M = 128 (two A blocks
// in 128-byte-swizzled shared memory), N = 128 (one B image), K = 64 per instruction, four
// instructions per 256-deep stage, scale factors in tensor memory, fp32 accumulators D0 / D1 in
// tensor memory.  The operands are zero (the tensor pipe's time does not depend on the values).
// The only wait is the final commit's mbarrier, bounded; on a timeout the status word says so.
#include "common.cuh"
#include "umma.cuh"

namespace nvmoe {
namespace {

constexpr int kStage = 55296;                     // A0 | A1 | B image | scales (as prefill_fp4)
constexpr int kOffA1 = 16384, kOffB = 32768;
constexpr uint32_t kTmD = 0, kTmSF = 256, kTmCols = 512;

__global__ void __launch_bounds__(128, 1) fp4_mma_probe(int n_iter, int32_t* status) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    unsigned char* sm = reinterpret_cast<unsigned char*>(
        (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    __shared__ uint64_t bar;
    __shared__ uint32_t tmem_base;
    const int warp = threadIdx.x >> 5;
    for (int i = threadIdx.x; i < kStage / 16; i += blockDim.x)
        reinterpret_cast<uint4*>(sm)[i] = make_uint4(0, 0, 0, 0);
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        mbar_init_fence();
    }
    if (warp == 0) umma::tmem_alloc(&tmem_base, kTmCols);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    const uint32_t tm = tmem_base;
    {   // zero scale factors: 64 columns from kTmSF, this warp's 32 lanes
        uint32_t z[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) z[i] = 0;
#pragma unroll
        for (int c = 0; c < 64; c += 16) umma::st_x16(umma::lane_addr(tm + kTmSF, warp, c), z);
        umma::wait_st();
    }
    umma::fence_smem_async();
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (threadIdx.x == 0) {
        const uint32_t sa = smem_u32(sm);
        const uint32_t idesc = umma::idesc_mxf4(128, 128);
        for (int it = 0; it < n_iter; ++it) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const uint32_t acc = (it == 0 && i == 0) ? 0u : 1u;
                const uint64_t bd = umma::smem_desc_sw128(sa + kOffB + 32 * i);
                const uint32_t sf = tm + kTmSF;
                umma::mma_mxf4(tm + kTmD, umma::smem_desc_sw128(sa + 32 * i), bd, idesc,
                               sf + 4 * i, sf + 32 + 4 * i, acc);
                umma::mma_mxf4(tm + kTmD + 128, umma::smem_desc_sw128(sa + kOffA1 + 32 * i), bd,
                               idesc, sf + 16 + 4 * i, sf + 32 + 4 * i, acc);
            }
        }
        umma::commit(&bar);
    }
    __syncwarp();
    const bool ok = mbar_wait_bounded(&bar, 0);
    if (!ok && threadIdx.x == 0 && status) atomicExch(status, NVMOE_ERR_TIMEOUT);
    umma::fence_before_sync();
    __syncthreads();
    umma::fence_after_sync();
    if (warp == 0) umma::tmem_dealloc(tm, kTmCols);
}

}  // namespace
}  // namespace nvmoe

extern "C" int nvmoe_probe_fp4_mma(int n_iter, int n_ctas, int32_t* status, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (n_iter <= 0 || n_ctas <= 0) return NVMOE_ERR_INVALID_ARG;
    int dev = 0, sms = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    NVMOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    if (n_ctas > sms) return NVMOE_ERR_INVALID_ARG;  // one CTA per SM (tensor memory, waits)
    // more shared memory than the stage needs, so that no two CTAs share an SM (each takes all
    // 512 tensor-memory columns)
    const int smem = 120 * 1024;
    NVMOE_CUDA_TRY(
        cudaFuncSetAttribute(fp4_mma_probe, cudaFuncAttributeMaxDynamicSharedMemorySize, smem));
    fp4_mma_probe<<<n_ctas, 128, smem, (cudaStream_t)stream>>>(n_iter, status);
    return cuda_status("fp4_mma_probe launch", cudaGetLastError());
}
