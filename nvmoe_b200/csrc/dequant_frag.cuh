// In-register dequantisers that produce m16n8k16 A fragments (f16) straight from packed
// slot-pool bytes.  The K index order inside a warp tile is a permutation chosen per format so
// that every lane loads whole 16-byte runs; the B operand (activations) is loaded with the same
// permutation, so the dot products are unchanged.
//
// Fragment convention (mma.m16n8k16.row.col, g = lane/4, q = lane%4): in one k16 step the lane
// holds A[g][c], A[g+8][c] for the four fragment columns c in {2q, 2q+1, 2q+8, 2q+9}; these map
// to four consecutive physical K values K0(q, step) + {0, 1, 2, 3}.  The B fragment of the lane
// (token g of the 8-token group) covers the same four K values.
#pragma once

#include "common.cuh"

namespace nvmoe {

// ------------------------------------------------------------------ NVFP4 (FTW banks)
// Warp K tile: 128 values; lane q owns K [32q, 32q+32) of it = 16 code bytes and 2 scale bytes
// per row; step s (0..7) covers K 32q + 4s + {0..3}.
struct FmtNvfp4 {
    static constexpr int kWarpTileK = 128;
    static constexpr int kSteps = 8;
    struct Row {
        uint4 codes;
        uint32_t scale2;  // f16x2 of the two scales of the 32 values (lo = first 16)
    };
    // base: row start of the codes; sbase: row start of the scales; k0: tile start (elements)
    __device__ __forceinline__ static void load(Row& r, const uint8_t* base, const uint8_t* sbase,
                                                int k0, int q) {
        r.codes = ldg_stream16(base + (k0 >> 1) + q * 16);
        r.scale2 = e4m3x2_to_f16x2(ldg_stream2(sbase + (k0 >> 4) + q * 2));
    }
    // same, from a shared-memory copy of the rows (staged by the TMA producer)
    __device__ __forceinline__ static void load_smem(Row& r, const uint8_t* base,
                                                     const uint8_t* sbase, int k0, int q) {
        r.codes = *reinterpret_cast<const uint4*>(base + (k0 >> 1) + q * 16);
        r.scale2 = e4m3x2_to_f16x2(*reinterpret_cast<const uint16_t*>(sbase + (k0 >> 4) + q * 2));
    }
    // bytes of one row of K values in the code / scale banks
    __host__ __device__ static constexpr int code_bytes(int k) { return k / 2; }
    __host__ __device__ static constexpr int scale_bytes(int k) { return k / 16; }
    // A values of step s: two f16x2 regs {K0, K0+1}, {K0+2, K0+3}.  The code word is split
    // into byte registers by a vector mov (no shift / mask per byte) and each byte converted
    // by cvt.rn.f16x2.e2m1x2; the scale multiply is exact (E2M1 x E4M3 fits f16).
    __device__ __forceinline__ static void deq(const Row& r, int s, uint32_t& lo, uint32_t& hi) {
        const uint32_t word = (&r.codes.x)[s >> 1];
        const uint32_t sc = (s < 4) ? prmt(r.scale2, 0, 0x1010) : prmt(r.scale2, 0, 0x3232);
        uint32_t a, b;
        if ((s & 1) == 0)
            asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
                "mov.b32 {b0, b1, b2, b3}, %2;\n\t"
                "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
                "cvt.rn.f16x2.e2m1x2 %1, b1; }"
                : "=r"(a), "=r"(b)
                : "r"(word));
        else
            asm("{ .reg .b8 b0, b1, b2, b3;\n\t"
                "mov.b32 {b0, b1, b2, b3}, %2;\n\t"
                "cvt.rn.f16x2.e2m1x2 %0, b2;\n\t"
                "cvt.rn.f16x2.e2m1x2 %1, b3; }"
                : "=r"(a), "=r"(b)
                : "r"(word));
        lo = hmul2_u32(a, sc);
        hi = hmul2_u32(b, sc);
    }
    // physical K offset (inside the warp tile) of step s for lane quarter q
    __device__ __forceinline__ static int kofs(int q, int s) { return 32 * q + 4 * s; }
};

}  // namespace nvmoe
