// Pieces shared by the block-scaled FP4 tensor-core kernels (decode FFN and prefill GEMMs):
// tensor maps over the NVFP4 slot banks, release / acquire counters with bounded waits, TMA
// loads, and the activation quantiser that turns rows of activations into NVFP4 terms in the
// 128-byte-swizzled K-major layout the MMA reads (B operand images).
#pragma once

#include <cuda.h>  // CUtensorMap and its enums (the encoder itself comes through the runtime)

#include "common.cuh"
#include "ffn_common.cuh"

namespace nvmoe {

// The six tensor maps of one pool: [gate codes, gate scales, up codes, up scales, down codes,
// down scales]; gate / up boxes are 64 rows (a gate_up tile stacks 64 gate over 64 up rows),
// down boxes 128 rows; codes 128 bytes wide (128-byte swizzle), scales 16 bytes.  Host side,
// cached per bank; false when a bank breaks the TMA rules (alignment, strides).
enum { M_GATE = 0, M_GATE_SF = 1, M_UP = 2, M_UP_SF = 3, M_DOWN = 4, M_DOWN_SF = 5 };
bool fp4_pool_maps(const nvmoe_expert_pool& p, CUtensorMap* m);

#ifdef __CUDACC__
namespace fp4 {

__device__ __forceinline__ int ld_acquire(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void fence_proxy_async_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, int x, int y, int z,
                                            uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// Bounded waits that also stop when another role of the CTA has given up (abort flag).
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, volatile int* abort) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        if (mbar_test_wait(bar, parity)) return true;
        if ((i & 63) == 63 && *abort) return false;
        if (i > 32) __nanosleep(i < 1024 ? 20 : 200);
    }
    *abort = 1;
    return false;
}
__device__ __forceinline__ bool wait_count(const int* p, int target, volatile int* abort) {
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        if (ld_acquire(p) >= target) return true;
        if ((i & 63) == 63 && *abort) return false;
        if (i > 16) __nanosleep(i < 1024 ? 32 : 200);
    }
    *abort = 1;
    return false;
}

// ---- activation quantisation: 16 values -> kFp4Terms x (8 bytes E2M1, 1 byte UE4M3)
__device__ __forceinline__ uint32_t e4m3_code(float v) {
    uint16_t r;
    asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
    return r & 0xffu;
}
__device__ __forceinline__ float e4m3_value(uint32_t code) {
    const uint32_t h2 = e4m3x2_to_f16x2((uint16_t)code);
    return __half2float(__ushort_as_half((uint16_t)(h2 & 0xffffu)));
}
// Byte offsets inside one stage of an operand image (npad rows): row n's 128 code bytes in the
// 128-byte swizzle (16-byte chunk c stored at chunk c ^ (n % 8)), then the rows' 16 scale bytes.
__device__ __forceinline__ int img_code_off(int n, int blk) {
    return n * 128 + ((((blk >> 1) ^ (n & 7))) << 4) + ((blk & 1) << 3);
}
__device__ __forceinline__ int img_sf_off(int npad, int n, int blk) {
    return npad * 128 + n * 16 + blk;
}
// Four consecutive lanes (q = lane & 3) quantise one 16-block, 4 values each: per term, the
// block maximum over the 4 lanes, a UE4M3 scale rounded up so the block fits (times
// 2^(ke + 2 t)), E2M1 round-to-nearest of the residual.  two[t] = this lane's 2 code bytes of
// term t, sc[t] = the term's scale byte (the same on the 4 lanes).  Called by all 32 lanes of
// the warp together.
__device__ __forceinline__ void quant4_terms(float (&v)[4], int ke, uint16_t (&two)[kFp4Terms],
                                             uint8_t (&sc)[kFp4Terms]) {
#pragma unroll
    for (int t = 0; t < kFp4Terms; ++t) {
        float am = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
        am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
        const float target = am * (1.0f / 6.0f) * fp4_exp2(ke + 2 * t);
        uint32_t code = e4m3_code(target);
        float sv = e4m3_value(code);
        if (sv < target && code < 0x7eu) sv = e4m3_value(++code);  // round the scale up
        const float s = sv * fp4_exp2(-(ke + 2 * t));
        const float inv = s > 0.f ? 1.0f / s : 0.f;
        uint16_t w;
        asm("{ .reg .b8 b0, b1;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
            "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
            "mov.b16 %0, {b0, b1}; }"
            : "=h"(w)
            : "f"(v[0] * inv), "f"(v[1] * inv), "f"(v[2] * inv), "f"(v[3] * inv));
        const uint32_t lo = e2m1x2_to_f16x2(w & 0xffu), hi = e2m1x2_to_f16x2(w >> 8);
        const float2 d01 = __half22float2(*reinterpret_cast<const __half2*>(&lo));
        const float2 d23 = __half22float2(*reinterpret_cast<const __half2*>(&hi));
        v[0] = fmaf(-d01.x, s, v[0]);
        v[1] = fmaf(-d01.y, s, v[1]);
        v[2] = fmaf(-d23.x, s, v[2]);
        v[3] = fmaf(-d23.y, s, v[3]);
        two[t] = w;
        sc[t] = (uint8_t)code;
    }
}
// The block's kFp4Terms rows 4 i + t into a stage of an image with npad rows (128-byte
// swizzle, scales after the npad code rows): this lane's 2 code bytes, lane q = 0 the scales.
__device__ __forceinline__ void put4(uint8_t* img, int npad, int i, int blk,
                                     const uint16_t (&two)[kFp4Terms], const uint8_t (&sc)[kFp4Terms]) {
    const int q = threadIdx.x & 3;
#pragma unroll
    for (int t = 0; t < kFp4Terms; ++t) {
        const int n = kFp4Terms * i + t;
        *reinterpret_cast<uint16_t*>(img + img_code_off(n, blk) + 2 * q) = two[t];
        if (q == 0) img[img_sf_off(npad, n, blk)] = sc[t];
    }
}

// quant4_terms, then the rows to a group image (npad > 0: put4) or to a token image (npad = 0:
// term row t of the stage's 512-byte row block, stored in both swizzle phases a token can take
// in a group (even or odd position), and the scales at byte offset i).  Lanes without a block
// pass active = false.
__device__ __forceinline__ void quant4_put(float (&v)[4], int ke, bool active, uint8_t* img,
                                           int npad, int i, int blk) {
    uint16_t two[kFp4Terms];
    uint8_t sc[kFp4Terms];
    quant4_terms(v, ke, two, sc);
    if (!active) return;
    if (npad > 0) {
        put4(img, npad, i, blk, two, sc);
        return;
    }
    const int q = threadIdx.x & 3;
#pragma unroll
    for (int t = 0; t < kFp4Terms; ++t) {
        const int off = ((blk & 1) << 3) + 2 * q;
        *reinterpret_cast<uint16_t*>(img + t * 128 + ((((blk >> 1) ^ t)) << 4) + off) = two[t];
        *reinterpret_cast<uint16_t*>(img + 512 + t * 128 + ((((blk >> 1) ^ (4 + t))) << 4) + off) = two[t];
        if (q == 0) img[i + t * 16 + blk] = sc[t];
    }
}

__device__ __forceinline__ int npad_of(int nt) { return (kFp4Terms * nt + 7) & ~7; }

// Contiguous per-CTA ranges of S items over G CTAs (S * (G + 1) < 2^32: 32-bit division).
__device__ __forceinline__ int range_lo(int S, int c, int G) {
    return (int)((uint32_t)c * (uint32_t)S / (uint32_t)G);
}

}  // namespace fp4
#endif  // __CUDACC__

}  // namespace nvmoe
