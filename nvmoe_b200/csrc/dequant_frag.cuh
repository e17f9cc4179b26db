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
    static constexpr int kAuxBytes = 0;  // no table in shared memory
    __device__ __forceinline__ static void load_smem(Row& r, const uint8_t* base,
                                                     const uint8_t* sbase, int k0, int q,
                                                     const uint32_t* aux = nullptr) {
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


// ------------------------------------------------------------------ bf16 rows
// [rows, K] bf16, no scale bank.  Lane quarter q owns the 32 values 32 q .. 32 q + 31 of a
// 128-wide warp tile (64 bytes); step s covers values 4 s .. 4 s + 3.  bf16 -> f16 is exact for
// magnitudes in the f16 normal range (bf16 has the shorter mantissa).
struct FmtBf16 {
    static constexpr int kWarpTileK = 128;
    static constexpr int kSteps = 8;
    static constexpr int kAuxBytes = 0;
    struct Row {
        uint4 v[4];
    };
    __device__ __forceinline__ static void load_smem(Row& r, const uint8_t* base,
                                                     const uint8_t*, int k0, int q,
                                                     const uint32_t* = nullptr) {
        const uint4* p = reinterpret_cast<const uint4*>(base + 2 * k0 + 64 * q);
#pragma unroll
        for (int i = 0; i < 4; ++i) r.v[i] = p[i];
    }
    __host__ __device__ static constexpr int code_bytes(int k) { return 2 * k; }
    __host__ __device__ static constexpr int scale_bytes(int) { return 0; }
    __device__ __forceinline__ static uint32_t to_f16x2(uint32_t w) {
        const __half2 h = __floats2half2_rn(__uint_as_float(w << 16), __uint_as_float(w & 0xffff0000u));
        return *reinterpret_cast<const uint32_t*>(&h);
    }
    __device__ __forceinline__ static void deq(const Row& r, int s, uint32_t& lo, uint32_t& hi) {
        const uint4 u = r.v[s >> 1];
        lo = to_f16x2((s & 1) ? u.z : u.x);
        hi = to_f16x2((s & 1) ? u.w : u.y);
    }
    __device__ __forceinline__ static int kofs(int q, int s) { return 32 * q + 4 * s; }
};

// ------------------------------------------------------------------ Q2_K (ggml block_q2_K)
// 84 B per 256 values: scales[16] (low nibble sc, high nibble m), qs[64], fp16 d, fp16 dmin;
// value e = 128 h + 32 j + 16 l16 + l (l < 16) is (qs[32 h + 16 l16 + l] >> 2 j) & 3 of
// sub-block 8 h + 2 j + l16, y = (d sc) q - dmin m.
// Warp K tile = one block.  Lane quarter q owns (h, l16) = (q >> 1, q & 1): its 16 qs bytes
// (4 words = byte groups l = 0..3, 4..7, ...) give 16 steps s = 4 j + word, each step 4 values
// of one sub-block.  Dequant in f16: the 2-bit integers exactly (prmt into 0x64xx = 1024 + q,
// minus 1024), then one fma with (d sc, -dmin m) rounded to f16.
struct FmtQ2K {
    static constexpr int kWarpTileK = 256;
    static constexpr int kSteps = 16;
    static constexpr int kAuxBytes = 0;
    struct Row {
        uint32_t qs[4];
        uint32_t dlml[4];  // f16x2 {d sc_j, -dmin m_j} for j = 0..3
    };
    __device__ __forceinline__ static void load_smem(Row& r, const uint8_t* base,
                                                     const uint8_t*, int k0, int q,
                                                     const uint32_t* = nullptr) {
        const uint8_t* blk = base + (k0 >> 8) * 84;  // 4-byte aligned
        const int h = q >> 1, l16 = q & 1;
        const uint32_t* qs = reinterpret_cast<const uint32_t*>(blk + 16 + 32 * h + 16 * l16);
#pragma unroll
        for (int i = 0; i < 4; ++i) r.qs[i] = qs[i];
        const uint32_t sw0 = *reinterpret_cast<const uint32_t*>(blk + 8 * h);
        const uint32_t sw1 = *reinterpret_cast<const uint32_t*>(blk + 8 * h + 4);
        const uint32_t dd = *reinterpret_cast<const uint32_t*>(blk + 80);
        const float d = __half2float(__ushort_as_half((unsigned short)(dd & 0xffff)));
        const float dmin = __half2float(__ushort_as_half((unsigned short)(dd >> 16)));
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const uint32_t sc = ((j < 2 ? sw0 : sw1) >> (8 * (l16 + 2 * (j & 1)))) & 0xff;
            const __half dl = __float2half_rn(d * (float)(sc & 15));
            const __half nml = __float2half_rn(-(dmin * (float)(sc >> 4)));
            r.dlml[j] = (uint32_t)__half_as_ushort(dl) | ((uint32_t)__half_as_ushort(nml) << 16);
        }
    }
    __host__ __device__ static constexpr int code_bytes(int k) { return k / 256 * 84; }
    __host__ __device__ static constexpr int scale_bytes(int) { return 0; }
    __device__ __forceinline__ static void deq(const Row& r, int s, uint32_t& lo, uint32_t& hi) {
        const int j = s >> 2;
        const uint32_t v = (r.qs[s & 3] >> (2 * j)) & 0x03030303u;
        const uint32_t k1024 = 0x64006400u;  // f16x2 {1024, 1024}
        const uint32_t dl = prmt(r.dlml[j], 0, 0x1010), nml = prmt(r.dlml[j], 0, 0x3232);
        lo = hfma2_u32(hsub2_u32(prmt(v, 0x64646464u, 0x4140), k1024), dl, nml);
        hi = hfma2_u32(hsub2_u32(prmt(v, 0x64646464u, 0x4342), k1024), dl, nml);
    }
    __device__ __forceinline__ static int kofs(int q, int s) {
        return 128 * (q >> 1) + 32 * (s >> 2) + 16 * (q & 1) + 4 * (s & 3);
    }
};

// ------------------------------------------------------------------ IQ2_XXS (ggml block_iq2_xxs)
// 66 B per 256 values: fp16 d, then per 32 values (group g) aux0 = 4 grid indices and aux1 =
// 4 x 7-bit sign indices | scale << 28; value 32 g + 8 l + i = db_g * grid[aux0.l][i] * sign,
// db_g = d (0.5 + scale) / 4, sign bit i of ksigns[(aux1 >> 7 l) & 127] (index | parity << 7).
// Warp K tile = one block.  Lane quarter q owns groups 2q, 2q + 1 (16 bytes); step
// s = 8 g' + 2 l + half covers grid bytes 4 half .. 4 half + 3 of entry l of group 2q + g'.
// The grid (256 x 8 magnitude bytes) is read from a shared-memory copy (aux).
struct FmtIQ2XXS {
    static constexpr int kWarpTileK = 256;
    static constexpr int kSteps = 16;
    static constexpr int kAuxBytes = 256 * 8;
    struct Row {
        uint32_t w[4];       // aux0, aux1 of group 2q, then of group 2q + 1
        uint32_t db;         // f16 db of the two groups (lo, hi)
        const uint32_t* grid;
    };
    __device__ __forceinline__ static void load_smem(Row& r, const uint8_t* base,
                                                     const uint8_t*, int k0, int q,
                                                     const uint32_t* aux = nullptr) {
        const uint8_t* blk = base + (k0 >> 8) * 66;  // 2-byte aligned
        const uint16_t* p = reinterpret_cast<const uint16_t*>(blk + 2 + 16 * q);
#pragma unroll
        for (int i = 0; i < 4; ++i) r.w[i] = (uint32_t)p[2 * i] | ((uint32_t)p[2 * i + 1] << 16);
        const float d = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
        const __half db0 = __float2half_rn(d * (0.5f + (float)(r.w[1] >> 28)) * 0.25f);
        const __half db1 = __float2half_rn(d * (0.5f + (float)(r.w[3] >> 28)) * 0.25f);
        r.db = (uint32_t)__half_as_ushort(db0) | ((uint32_t)__half_as_ushort(db1) << 16);
        r.grid = aux;
    }
    __host__ __device__ static constexpr int code_bytes(int k) { return k / 256 * 66; }
    __host__ __device__ static constexpr int scale_bytes(int) { return 0; }
    __device__ __forceinline__ static void deq(const Row& r, int s, uint32_t& lo, uint32_t& hi) {
        const int g = s >> 3, l = (s >> 1) & 3, half = s & 1;
        const uint32_t a0 = r.w[2 * g], a1 = r.w[2 * g + 1];
        const uint32_t gw = r.grid[((a0 >> (8 * l)) & 0xff) * 2 + half];  // 4 magnitudes
        const uint32_t si = (a1 >> (7 * l)) & 127;
        const uint32_t sb = (si | ((uint32_t)(__popc(si) & 1) << 7)) >> (4 * half);
        const uint32_t k1024 = 0x64006400u;
        const uint32_t mlo = hsub2_u32(prmt(gw, 0x64646464u, 0x4140), k1024);
        const uint32_t mhi = hsub2_u32(prmt(gw, 0x64646464u, 0x4342), k1024);
        // sign bits i -> f16 sign bits (bit 15 of the low half, bit 31 of the high half)
        const uint32_t slo = ((sb & 1u) << 15) | ((sb & 2u) << 30);
        const uint32_t shi = ((sb & 4u) << 13) | ((sb & 8u) << 28);
        const uint32_t db = g ? prmt(r.db, 0, 0x3232) : prmt(r.db, 0, 0x1010);
        lo = hmul2_u32(mlo ^ slo, db);
        hi = hmul2_u32(mhi ^ shi, db);
    }
    __device__ __forceinline__ static int kofs(int q, int s) {
        return 64 * q + 32 * (s >> 3) + 8 * ((s >> 1) & 3) + 4 * (s & 1);
    }
};

}  // namespace nvmoe
