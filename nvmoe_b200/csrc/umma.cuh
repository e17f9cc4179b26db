// 5th-generation tensor core (tcgen05) building blocks for sm_100a: TMEM allocation, MMA issue
// with A in shared or tensor memory, completion through an mbarrier, and TMEM <-> register
// moves.  Layout conventions used by every caller of this header:
//
//   * Operands in shared memory are K-major, no swizzle, in the canonical "core matrix" layout:
//     a core matrix is 8 rows x 16 bytes (8 f16 of K) stored contiguously (128 B); for a tile of
//     `rows` rows the core matrix of row group rg and K group kc sits at
//     ((kc * rows / 8) + rg) * 128 bytes.  One MMA K-step (16 f16) then has LBO = rows / 8 * 128
//     (between its two K groups) and SBO = 128 (between row groups).
//   * A in tensor memory (M = 128): row r in TMEM lane r, two f16 per 32-bit column, lower K in
//     the low half; one K-step is 8 columns.
//   * D (fp32, M = 128): row r in lane r, column n in TMEM column base + n.
//   * A warp can only touch TMEM lanes 32 * (warp % 4) .. + 31.
#pragma once

#include "common.cuh"

namespace nvmoe {
namespace umma {

__device__ __forceinline__ int canon_off(int r, int k, int rows) {
    return (((k >> 3) * (rows >> 3) + (r >> 3)) * 128) + (r & 7) * 16 + (k & 7) * 2;
}

// Shared-memory matrix descriptor: start / leading / stride byte offsets (16-byte units),
// descriptor version 1 (sm_100), base offset 0, no swizzle.
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    return d;
}

// Instruction descriptor of kind::f16 with f16 A and B, fp32 accumulate, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols));
}
__device__ __forceinline__ void fence_before_sync() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// generic-proxy shared-memory writes -> visible to the tensor core
__device__ __forceinline__ void fence_smem_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// D (+)= A * B^T, A and B from shared memory.
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// D (+)= A * B^T, A from tensor memory, B from shared memory.
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate));
}
// Arrive on an mbarrier once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void commit(uint64_t* bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
        "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void ld_x16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
          "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]),
          "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr)
        : "memory");
}
// Shared-memory descriptor of a K-major tile in the 128-byte swizzle layout that TMA writes with
// CU_TENSOR_MAP_SWIZZLE_128B: 128-byte rows, 8-row (1024-byte) swizzle atoms stacked along M/N
// (SBO = 1024; LBO unused).  The tile base must be 1024-byte aligned; a K step inside the
// 128-byte row advances the start address (32 bytes per 64 FP4 values).
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t addr) {
    uint64_t d = 0;
    d |= (uint64_t)((addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor of kind::mxf4nvf4: A and B E2M1 (packed, two per byte), UE4M3 scale
// factors, K-major, dense K = 64 per instruction, fp32 accumulate.
__host__ __device__ constexpr uint32_t idesc_mxf4(int m, int n) {
    return (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// D (+)= (A x SFA) * (B x SFB)^T, K = 64, one UE4M3 scale per 16 values of each row of A and B.
// Scale factors in tensor memory (column addresses 4-column aligned):
//   SFA (M = 128): column sfa + m1, lane m0 (and the same in the other three lane quadrants)
//                  hold the 4 scales of row 32 m1 + m0, K block j in byte j;
//   SFB (N <= 32): column sfb, lane n (every quadrant) holds the 4 scales of row n.
__device__ __forceinline__ void mma_mxf4(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t sfa_tmem, uint32_t sfb_tmem,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], "
        "[%6], p;\n\t}" ::"r"(d_tmem),
        "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate), "r"(sfa_tmem), "r"(sfb_tmem));
}

__device__ __forceinline__ void wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// TMEM address of column `col` in the lanes of this warp's quadrant.
__device__ __forceinline__ uint32_t lane_addr(uint32_t base, int warp, int col) {
    return base + ((uint32_t)((warp & 3) * 32) << 16) + (uint32_t)col;
}

}  // namespace umma
}  // namespace nvmoe
