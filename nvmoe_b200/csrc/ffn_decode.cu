// R7 / R9 — routed-expert FFN over the slot pool for decode-sized batches.
//
// Reference call: _expert_gemm(cache, hidden, topk_weights, slot_ids, views, n, alphas,
// is_prefill) (nvme-moe-bench/nvme_offload_cache.py:1989-1998, 2165-2174) and ggml mul_mat_id
// over the reduced [.., .., cache_size] expert tensors (scripts/test_mul_mat_id_shrink.cpp:29-69):
//   y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] ),  s = slot_ids[t, j]
// plus the always-on shared expert (nvme_offload_cache.py:2115-2123).
//
// Kernels (chained with programmatic dependent launch):
//   prep  — x -> f16, shared-expert gate, grouping of the (token, k) entries by slot into token
//           groups of <= 8 entries with complete group records (ffn_common.cuh); the fused
//           decode front kernel does the same work in the engine path
//   fused — persistent, one CTA per SM, warp-specialised: a producer warp streams gate_up work
//           items (token group x 16 rows of gate and of up) and then down slabs (16 rows of a
//           CTA's output tile for every group) with 1-D bulk copies (TMA) into two rings of
//           shared-memory stages; 8 MMA warps dequantise A fragments in registers from the
//           staged bytes and run m16n8k16 f16 MMAs (fp32 accumulate); an epilogue warp sums the
//           gate_up partials of the 8 warps, stores h = silu(g) * u (f16) and publishes each
//           finished row tile on a per-group counter; the down phase starts a group once its
//           counter is complete, writes w * down(h) per entry into shared memory, and each CTA
//           finally sums the entries of each token in the fixed order j = 0..k-1, shared, and
//           stores bf16 y.  No atomics on data, deterministic.
// Only the slots that occur in slot_ids are read; every weight byte is read once per call.
#include "common.cuh"
#include "dequant_frag.cuh"
#include "ffn_common.cuh"

#include <algorithm>

namespace nvmoe {

// IQ2_XXS grid registered with nvmoe_set_iq2xxs_grid (dequant.cu)
bool iq2xxs_grid_ready(int device);
const uint8_t* iq2xxs_grid_device_ptr();

namespace {

constexpr int kConsumerWarps = 8;
constexpr int kConsumers = kConsumerWarps * 32;
constexpr int kSmemCap = 227 * 1024 - 1024;   // dynamic share; static use stays below 1 KB
// x rows in a gate_up stage are kXPad bytes apart beyond their length, so the 8 token rows of
// a B-fragment load fall into different shared-memory banks
constexpr int kXPad = 16;
constexpr int kStageHdr = 128;  // per stage: a copy of the group record (kDescInts ints)

// ------------------------------------------------------------------ 1. prep
__global__ void __launch_bounds__(kPrepThreads) ffn_prep_kernel(FfnParams P) {
    extern __shared__ __align__(16) int prep_smem[];
    grid_dep_wait();
    grid_dep_launch();
    if ((int)blockIdx.x < (int)gridDim.x - 1) {
        ffn_convert_tokens(P, blockIdx.x, gridDim.x - 1);
    } else {
        ffn_group_block(P, prep_smem);
    }
}

__device__ __forceinline__ void report_timeout(const FfnParams& P) {
    atomicExch(wsp<int>(P, P.L.hdr) + HDR_STATUS, NVMOE_ERR_TIMEOUT);
    if (P.status) atomicExch(P.status, NVMOE_ERR_TIMEOUT);
}

// ------------------------------------------------------------------ in-kernel refill
// The misses of a decode layer step are copied from the pinned host tier by one warp of every
// CTA while the other warps run the hit groups (the grouping orders missed groups last); each
// piece ends with a release on the miss's counter, and a producer about to stage a missed
// slot's rows acquires it first.  Generic-proxy stores read later by bulk copies (async proxy):
// a proxy fence on both sides.
__device__ __forceinline__ void proxy_fence_global() {
    asm volatile("fence.proxy.async.global;" ::: "memory");
}
__device__ __forceinline__ void refill_pieces(const FfnParams& P, int lane) {
    const FfnRefill& R = P.rf;
    const int ppm = R.pbase[R.n_banks];
    const int n_miss = __ldcg(R.counts + 1);
    int* rdy = wsp<int>(P, P.L.rdy);
    for (int p = blockIdx.x; p < n_miss * ppm; p += gridDim.x) {
        const int m = p / ppm, q = p - m * ppm;
        int b = 0;
        while (b + 1 < R.n_banks && q >= R.pbase[b + 1]) ++b;
        const nvmoe_refill_bank& B = R.banks[b];
        const int gs = __ldcg(R.miss_slots + m);
        const int id = __ldcg(R.miss_ids + m);
        const int hs = id >= 0 ? __ldcg(R.host_slot_of_id + id) : -1;
        if (hs < 0 || gs < 0 || gs >= R.n_gpu_slots) {
            if (lane == 0) atomicExch(R.counts + 2, NVMOE_ERR_HOST_LOAD);
        } else {
            const int64_t beg = (int64_t)(q - R.pbase[b]) * kRefillPiece;
            const int len = (int)min((int64_t)kRefillPiece, B.row_bytes - beg);
            const char* src = static_cast<const char*>(B.src) + (int64_t)hs * B.src_slot_stride + beg;
            char* dst = static_cast<char*>(B.dst) + (int64_t)gs * B.dst_slot_stride + beg;
            if (R.vec16[b]) {  // all of a piece's loads in flight at once (PCIe latency)
                const uint4* s16 = reinterpret_cast<const uint4*>(src);
                uint4* d16 = reinterpret_cast<uint4*>(dst);
                const int n16 = len >> 4;
                uint4 v[kRefillPiece / 16 / 32];
#pragma unroll
                for (int i = 0; i < kRefillPiece / 16 / 32; ++i)
                    if (lane + 32 * i < n16) v[i] = s16[lane + 32 * i];
#pragma unroll
                for (int i = 0; i < kRefillPiece / 16 / 32; ++i)
                    if (lane + 32 * i < n16) d16[lane + 32 * i] = v[i];
            } else if (R.vec4[b]) {  // e.g. the fp32 global-scale bank
                for (int i = lane; i < (len >> 2); i += 32)
                    reinterpret_cast<uint32_t*>(dst)[i] = reinterpret_cast<const uint32_t*>(src)[i];
            } else {
                for (int i = lane; i < len; i += 32) dst[i] = src[i];
            }
        }
        proxy_fence_global();
        __threadfence();
        __syncwarp();
        if (lane == 0)  // also after a bad slot, so that no waiter runs into its limit
            asm volatile("red.release.gpu.global.add.s32 [%0], 1;" ::"l"(rdy + 2 * m + R.down[b])
                         : "memory");
    }
}
// Whether missed slot mi's gate/up banks (down = 0) or all its banks (down = 1) are in; after a
// true result the caller's bulk copies see them.
__device__ __forceinline__ bool refill_ready(const FfnParams& P, int mi, int down) {
    const int* c = wsp<int>(P, P.L.rdy) + 2 * mi;
    int v0, v1 = 0;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v0) : "l"(c) : "memory");
    if (down) asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v1) : "l"(c + 1) : "memory");
    if (v0 >= P.rf.pieces_gu && (!down || v1 >= P.rf.pieces_dn)) {
        proxy_fence_global();
        return true;
    }
    return false;
}
// A producer's wait for missed slot mi (bounded): the gate/up banks (down = 0), or every bank
// (down = 1; a bank the host did not recognise as a down bank counts with the gate/up ones).
__device__ __forceinline__ bool refill_wait(const FfnParams& P, int mi, int down) {
    const int* c = wsp<int>(P, P.L.rdy) + 2 * mi;
    for (uint32_t i = 0; i < (1u << 24); ++i) {
        int v0, v1 = 0;
        asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v0) : "l"(c) : "memory");
        if (down) asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v1) : "l"(c + 1) : "memory");
        if (v0 >= P.rf.pieces_gu && (!down || v1 >= P.rf.pieces_dn)) {
            proxy_fence_global();
            return true;
        }
        if (i > 16) __nanosleep(i < 1024 ? 64 : 256);
    }
    return false;
}

// Copies `rows` rows of `row_bytes` from a bank (row stride `stride`) into contiguous smem.
__device__ __forceinline__ void bulk_rows(uint8_t* dst, const uint8_t* src, int rows,
                                          int row_bytes, int64_t stride, uint64_t* bar) {
    const uint64_t pol = l2_evict_first_policy();
    if (stride == row_bytes) {
        bulk_g2s_stream(dst, src, (uint32_t)(rows * row_bytes), bar, pol);
    } else {
        for (int r = 0; r < rows; ++r)
            bulk_g2s_stream(dst + r * row_bytes, src + r * stride, (uint32_t)row_bytes, bar, pol);
    }
}

// ------------------------------------------------------------------ 2. fused gate_up + down
// Shared memory: [gate_up ring][resident x][down ring][red: 2 x 8 warps x 32 lanes x 8
// floats][meta: 2 x 8 ints][y_part (optional)][mbarriers].  Once the gate_up phase has drained,
// its ring's bytes hold further down stages.
//   gate_up stage: [record 128 B] gate codes [16][H/2] | up codes | gate scales [16][H/16] |
//                  up scales | x [XT][H + 8] f16 when x is staged per item (XT = the largest
//                  group of this launch; the 8 extra halves per row only spread the rows over
//                  the banks); resident x: [n_tok][H + 8] f16 once per CTA (n_tok <= 8)
//   down stage   : [record 128 B] codes [16][I/2] | scales [16][I/16]
struct FusedLayout {
    int stage_gu, stage_dn;  // bytes per stage
    int nst_gu;              // gate_up ring stages
    int nst_dn;              // down stages in their own region (a multiple of 8)
    int nst_dn_ext;          // down stages carved from the gate_up ring once it has drained
    int xt;                  // x rows per gate_up stage (staged x), 0 with resident x
    int x_res;               // 1: every token row resident in shared memory, loaded once
    int off_x, off_dn, off_red, off_meta, off_yp, off_bar, total;
    int off_aux;             // the format's lookup table (IQ2_XXS grid)
};

__host__ __device__ inline int round128(int v) { return (v + 127) / 128 * 128; }

// One 128-wide K tile of a 16-row gate + up item: rows g and g + 8 of both matrices for the
// lane quarter q, B = the activations of the group's tokens (token g of the lane).
// The MMAs of consecutive steps go to kAcc independent accumulators (a single accumulator
// chains every mma.sync on the previous one's result and leaves the warp latency-bound); the
// accumulators are summed in a fixed order at the end of the item.
constexpr int kAcc = 8;

template <typename Fmt>
__device__ __forceinline__ void gate_up_tile(const uint8_t* gcode, const uint8_t* ucode,
                                             const uint8_t* gsc, const uint8_t* usc, int cb,
                                             int sb, const uint32_t* aux, const __half* xs,
                                             bool has_tok, int k0,
                                             int g, int q, float (&accg)[kAcc][4],
                                             float (&accu)[kAcc][4]) {
    typename Fmt::Row ga, gb, ua, ub;
    Fmt::load_smem(ga, gcode + g * cb, gsc + g * sb, k0, q, aux);
    Fmt::load_smem(gb, gcode + (g + 8) * cb, gsc + (g + 8) * sb, k0, q, aux);
    Fmt::load_smem(ua, ucode + g * cb, usc + g * sb, k0, q, aux);
    Fmt::load_smem(ub, ucode + (g + 8) * cb, usc + (g + 8) * sb, k0, q, aux);
#pragma unroll
    for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
        const uint4 xb = has_tok ? *reinterpret_cast<const uint4*>(xs + k0 + Fmt::kofs(q, s2))
                                 : make_uint4(0, 0, 0, 0);
#pragma unroll
        for (int ss = 0; ss < 2; ++ss) {
            uint32_t ag[4], au[4];
            Fmt::deq(ga, s2 + ss, ag[0], ag[2]);
            Fmt::deq(gb, s2 + ss, ag[1], ag[3]);
            Fmt::deq(ua, s2 + ss, au[0], au[2]);
            Fmt::deq(ub, s2 + ss, au[1], au[3]);
            const uint32_t b0 = ss ? xb.z : xb.x, b1 = ss ? xb.w : xb.y;
            mma_f16_16816(accg[(s2 + ss) % kAcc], ag, b0, b1);
            mma_f16_16816(accu[(s2 + ss) % kAcc], au, b0, b1);
        }
    }
}

// One 128-wide K tile of a 16-row down slab: rows g and g + 8; hb = the lane's h fragments of
// this tile (4 x 8 halves of token g).
template <typename Fmt>
__device__ __forceinline__ void down_tile(const uint8_t* code, const uint8_t* sc, int cb, int sb,
                                          const uint32_t* aux, const uint4 (&hb)[Fmt::kSteps / 2],
                                          int k0, int g,
                                          int q, float (&acc)[kAcc][4]) {
    typename Fmt::Row ra, rbw;
    Fmt::load_smem(ra, code + g * cb, sc + g * sb, k0, q, aux);
    Fmt::load_smem(rbw, code + (g + 8) * cb, sc + (g + 8) * sb, k0, q, aux);
#pragma unroll
    for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
        const uint4 h = hb[s2 >> 1];
#pragma unroll
        for (int ss = 0; ss < 2; ++ss) {
            uint32_t af[4];
            Fmt::deq(ra, s2 + ss, af[0], af[2]);
            Fmt::deq(rbw, s2 + ss, af[1], af[3]);
            mma_f16_16816(acc[(s2 + ss) % kAcc], af, ss ? h.z : h.x, ss ? h.w : h.y);
        }
    }
}

// Sum of the kAcc accumulators (fixed order) into acc[0].
__device__ __forceinline__ void fold_acc(float (&acc)[kAcc][4]) {
#pragma unroll
    for (int a = 1; a < kAcc; ++a)
#pragma unroll
        for (int v = 0; v < 4; ++v) acc[0][v] += acc[a][v];
}

// h fragments of one K tile for token row hrow (null: no token -> zeros), in the order of the
// format's step pairs, read through L2 (h is written by other CTAs of this grid).
template <typename Fmt>
__device__ __forceinline__ void load_h_tile(const __half* hrow, int k0, int q,
                                            uint4 (&hb)[Fmt::kSteps / 2]) {
#pragma unroll
    for (int i = 0; i < Fmt::kSteps / 2; ++i)
        hb[i] = hrow ? __ldcg(reinterpret_cast<const uint4*>(hrow + k0 + Fmt::kofs(q, 2 * i)))
                     : make_uint4(0, 0, 0, 0);
}

__device__ __forceinline__ int ld_acquire_gpu(const int* p) {
    int v;
    asm volatile("ld.acquire.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
    asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Bounded wait until the group's h rows are complete (all I/16 gate/up row tiles stored).

__device__ __forceinline__ void copy_record(int* dst, const int4 (&r)[kDescInts / 4]) {
#pragma unroll
    for (int k = 0; k < kDescInts / 4; ++k) reinterpret_cast<int4*>(dst)[k] = r[k];
}
__device__ __forceinline__ void load_record(const FfnParams& P, int grp, int4 (&r)[kDescInts / 4]) {
    const int4* src = reinterpret_cast<const int4*>(wsp<int>(P, P.L.grp_desc) +
                                                    (int64_t)grp * kDescInts);
#pragma unroll
    for (int k = 0; k < kDescInts / 4; ++k) r[k] = __ldcg(src + k);
}
__device__ __forceinline__ void shfl_record(int4 (&dst)[kDescInts / 4],
                                            const int4 (&src)[kDescInts / 4], int lane) {
#pragma unroll
    for (int k = 0; k < kDescInts / 4; ++k) {
        dst[k].x = __shfl_sync(0xffffffffu, src[k].x, lane);
        dst[k].y = __shfl_sync(0xffffffffu, src[k].y, lane);
        dst[k].z = __shfl_sync(0xffffffffu, src[k].z, lane);
        dst[k].w = __shfl_sync(0xffffffffu, src[k].w, lane);
    }
}

constexpr int kCW = kConsumerWarps;       // MMA warps
constexpr int kProdGU = kCW;              // bulk-copy producer of the gate_up items
constexpr int kEpiWarp = kCW + 1;         // gate/up cross-warp sum + SwiGLU + h store
constexpr int kProdDN = kCW + 2;          // bulk-copy producer of the down slabs
constexpr int kRefillWarp = kCW + 3;      // copies this call's misses in from the host tier
constexpr int kFusedThreads = (kCW + 4) * 32;

// Persistent expert FFN, one CTA per SM.  CTA c runs
//   gate_up items c, c + G, ... (item = token group x 16 rows of gate and of up, full K = H),
//   then down row tiles r = G - 1 - c, 2G - 1 - c, ... (16 rows of y over every group, K = I).
// Roles: two producer warps stream the two phases' weights into their rings (down weights do
// not depend on h, so they are in flight while gate_up runs); the 8 MMA warps split K of a
// gate_up item (TPW tiles each, straight-line code) and hand their partial sums to the
// epilogue warp through a 2-deep ring, so they never wait for the cross-warp sum; the epilogue
// warp stores h and counts the group's finished row tiles (release); a down MMA warp owns whole
// groups and starts a group once its count is complete (acquire).
template <typename Fmt, int TPW, int TD>
__global__ void __launch_bounds__(kFusedThreads, 1) ffn_fused(FfnParams P, FusedLayout FL) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int G = gridDim.x;
    // (the down producer gives each ring stage to one lane: at most 32 stages are used)
    const int NGU = FL.nst_gu, NDT = min(FL.nst_dn + FL.nst_dn_ext, 32);
    uint64_t* gu_full = reinterpret_cast<uint64_t*>(smem + FL.off_bar);
    uint64_t* gu_empty = gu_full + NGU;
    uint64_t* dn_full = gu_empty + NGU;
    uint64_t* dn_empty = dn_full + NDT;
    uint64_t* red_full = dn_empty + NDT;
    uint64_t* red_empty = red_full + 2;
    uint64_t* x_full = red_empty + 2;
    uint64_t* gu_drained = x_full + 1;
    float* red = reinterpret_cast<float*>(smem + FL.off_red);
    int* meta = reinterpret_cast<int*>(smem + FL.off_meta);
    if (tid == 0) {
        for (int s = 0; s < NGU; ++s) mbar_init(&gu_full[s], 1), mbar_init(&gu_empty[s], kCW);
        for (int s = 0; s < NDT; ++s) mbar_init(&dn_full[s], 1), mbar_init(&dn_empty[s], 1);
        for (int s = 0; s < 2; ++s) mbar_init(&red_full[s], kCW), mbar_init(&red_empty[s], 1);
        mbar_init(x_full, 1);
        mbar_init(gu_drained, kCW);
        mbar_init_fence();
    }
    // the format's lookup table (IQ2_XXS grid), constant across calls
    uint32_t* aux = reinterpret_cast<uint32_t*>(smem + FL.off_aux);
    for (int i = tid; i < Fmt::kAuxBytes / 4; i += blockDim.x) aux[i] = __ldg(P.aux_table + i);
    __syncthreads();
    // everything below reads the group records / token rows of the kernel before this one
    grid_dep_wait();
    grid_dep_launch();

    const int tiles_i = I / 16, n_dn = H / 16;
    const int cbg = Fmt::code_bytes(H), sbg = Fmt::scale_bytes(H);
    const int cbd = Fmt::code_bytes(I), sbd = Fmt::scale_bytes(I);
    const int og_uc = kStageHdr + 16 * cbg, og_gs = kStageHdr + 32 * cbg;
    const int og_us = og_gs + 16 * sbg, og_x = og_us + 16 * sbg;
    const int od_sc = kStageHdr + 16 * cbd;
    const int xrow = H * 2 + kXPad;  // bytes between x rows in shared memory
    const __half* x16 = wsp<__half>(P, P.L.x16);
    __half* h16 = wsp<__half>(P, P.L.h16);
    int* done = wsp<int>(P, P.L.grp_done);
    const int* hdr_g = wsp<int>(P, P.L.hdr);
    // down stage st: its own region first, then the drained gate_up ring
    auto dn_stage = [&](int st) -> uint8_t* {
        return st < FL.nst_dn ? smem + FL.off_dn + (size_t)st * FL.stage_dn
                              : smem + (size_t)(st - FL.nst_dn) * FL.stage_dn;
    };

    if (warp == kRefillWarp) {
        if (P.rf.n_banks > 0) refill_pieces(P, lane);
        return;
    }

    if (warp == kProdGU) {
        // the first batch of records is fetched together with the group count (speculative
        // group indices, clamped into the workspace)
        int4 rec[kDescInts / 4];
        load_record(P, min((int)(blockIdx.x + lane * G) / tiles_i, P.L.g_max - 1), rec);
        const int n_groups = __ldcg(hdr_g + HDR_N_GROUPS);
        const int n_gu = n_groups * tiles_i;
        if (FL.x_res && lane == 0 && n_gu > (int)blockIdx.x) {
            mbar_arrive_expect_tx(x_full, (uint32_t)(P.n_tok * H * 2));
            for (int t = 0; t < P.n_tok; ++t)
                bulk_g2s(smem + FL.off_x + t * xrow, x16 + (int64_t)t * H, (uint32_t)(H * 2), x_full);
        }
        bool ok = true;
        int it = 0;
        for (int base = blockIdx.x; base < n_gu && ok; base += 32 * G) {
            const int mine = base + lane * G;
            if (base != (int)blockIdx.x && mine < n_gu) load_record(P, mine / tiles_i, rec);
            const int n_here = min(32, (n_gu - base + G - 1) / G);
            for (int i = 0; i < n_here; ++i, ++it) {
                int4 r[kDescInts / 4];
                shfl_record(r, rec, i);
                if (lane == 0) {
                    const int item = base + i * G;
                    const int st = it % NGU;
                    if (!mbar_wait_bounded(&gu_empty[st], ((it / NGU) & 1) ^ 1)) {
                        report_timeout(P);
                        ok = false;
                    } else {
                        uint8_t* stg = smem + (size_t)st * FL.stage_gu;
                        int* hdr = reinterpret_cast<int*>(stg);
                        copy_record(hdr, r);
                        if (hdr[GD_MISS] > 0 && !refill_wait(P, hdr[GD_MISS] - 1, 0)) {
                            report_timeout(P);
                            ok = false;
                        }
                        hdr[GD_RT] = item % tiles_i;
                        hdr[GD_GID] = item / tiles_i;
                        const nvmoe_expert_pool& pool = hdr[GD_POOL] ? P.shared : P.pool;
                        const int slot = hdr[GD_SLOT], nt = hdr[GD_NT];
                        const int64_t r0 = (int64_t)(item % tiles_i) * 16;
                        mbar_arrive_expect_tx(
                            &gu_full[st],
                            (uint32_t)(32 * cbg + 32 * sbg + (FL.x_res ? 0 : nt * H * 2)));
                        bulk_rows(stg + kStageHdr,
                                  (const uint8_t*)pool.gate.data + slot * pool.gate.slot_stride +
                                      r0 * pool.gate.row_stride,
                                  16, cbg, pool.gate.row_stride, &gu_full[st]);
                        bulk_rows(stg + og_uc,
                                  (const uint8_t*)pool.up.data + slot * pool.up.slot_stride +
                                      r0 * pool.up.row_stride,
                                  16, cbg, pool.up.row_stride, &gu_full[st]);
                        if (sbg > 0) {  // formats with a separate scale bank
                            bulk_rows(stg + og_gs,
                                      (const uint8_t*)pool.gate.scale +
                                          slot * pool.gate.scale_slot_stride +
                                          r0 * pool.gate.scale_row_stride,
                                      16, sbg, pool.gate.scale_row_stride, &gu_full[st]);
                            bulk_rows(stg + og_us,
                                      (const uint8_t*)pool.up.scale +
                                          slot * pool.up.scale_slot_stride +
                                          r0 * pool.up.scale_row_stride,
                                      16, sbg, pool.up.scale_row_stride, &gu_full[st]);
                        }
                        if (!FL.x_res)
                            for (int n = 0; n < nt; ++n)
                                bulk_g2s(stg + og_x + n * xrow, x16 + (int64_t)hdr[GD_TOK + n] * H,
                                         (uint32_t)(H * 2), &gu_full[st]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) break;
            }
        }
        return;
    }

    if (warp == kProdDN) {
        // down slabs: for each of this CTA's row tiles, every group's 16 rows; use j of the ring
        // is (row tile j / n_groups, group j % n_groups) in stage j % NDT.  Lane i owns stage i
        // and runs its uses i, i + NDT, ... as a state machine of its own, polled without
        // blocking (a lane that waited in a loop of its own would hold the others back):
        //   the gate_up ring drained (stages in its bytes) -> stage free -> missed slot's banks
        //   in -> rows requested (expect_tx, bulk copies) -> the group's h complete: down global
        //   scale and shared-expert gates into the stage's record copy, arrive (the MMA warp
        //   reads h without an acquire of its own: release -> acquire here, then the barrier)
        enum { S_DRAIN, S_FREE, S_REFILL, S_ISSUE, S_H, S_DONE };
        const int n_groups = __ldcg(hdr_g + HDR_N_GROUPS);
        const float* sgate = (P.has_shared && P.shared_gate) ? wsp<float>(P, P.L.sg) : nullptr;
        const int rt0 = G - 1 - (int)blockIdx.x;
        const int n_rt = rt0 < n_dn ? (n_dn - 1 - rt0) / G + 1 : 0;
        const int total = n_rt * n_groups;
        int j = lane;
        int state = (lane >= NDT || j >= total) ? S_DONE : (lane >= FL.nst_dn ? S_DRAIN : S_FREE);
        uint8_t* stg = dn_stage(lane < NDT ? lane : 0);
        int* hdr = reinterpret_cast<int*>(stg);
        int4 r[kDescInts / 4];
        if (state != S_DONE) load_record(P, j % n_groups, r);
        float dgl = 1.f;
        bool ok = true;
        for (uint32_t w = 0; __any_sync(0xffffffffu, state != S_DONE); ++w) {
            if (w == (1u << 24)) {  // about a second: give up
                if (state != S_DONE) {
                    report_timeout(P);
                    ok = false;
                }
                break;
            }
            if (state == S_DRAIN && mbar_test_wait(gu_drained, 0)) state = S_FREE;
            if (state == S_FREE && mbar_test_wait(&dn_empty[lane], ((j / NDT) & 1) ^ 1)) {
                copy_record(hdr, r);
                hdr[GD_GID] = j % n_groups;
                state = hdr[GD_MISS] > 0 ? S_REFILL : S_ISSUE;
            }
            if (state == S_REFILL && refill_ready(P, hdr[GD_MISS] - 1, 1)) state = S_ISSUE;
            if (state == S_ISSUE) {
                const nvmoe_expert_pool& pool = hdr[GD_POOL] ? P.shared : P.pool;
                const int slot = hdr[GD_SLOT];
                const int64_t r0 = (int64_t)(rt0 + (j / n_groups) * G) * 16;
                dgl = global_of_early(pool.down, slot);
                mbar_expect_tx(&dn_full[lane], (uint32_t)(16 * (cbd + sbd)));
                bulk_rows(stg + kStageHdr,
                          (const uint8_t*)pool.down.data + slot * pool.down.slot_stride +
                              r0 * pool.down.row_stride,
                          16, cbd, pool.down.row_stride, &dn_full[lane]);
                if (sbd > 0)
                    bulk_rows(stg + od_sc,
                              (const uint8_t*)pool.down.scale + slot * pool.down.scale_slot_stride +
                                  r0 * pool.down.scale_row_stride,
                              16, sbd, pool.down.scale_row_stride, &dn_full[lane]);
                state = S_H;
            }
            if (state == S_H && ld_acquire_gpu(done + j % n_groups) >= tiles_i) {
                hdr[GD_DGLOB] = __float_as_int(dgl);
                if (hdr[GD_POOL] && sgate) {
                    const int nt = hdr[GD_NT];
                    for (int k = 0; k < nt; ++k)
                        hdr[GD_W + k] = __float_as_int(__ldcg(sgate + hdr[GD_TOK + k]));
                }
                mbar_arrive(&dn_full[lane]);
                j += NDT;
                state = S_DONE;
                if (j < total) {
                    load_record(P, j % n_groups, r);  // (used once the stage is free again)
                    state = S_FREE;
                }
            }
            if (w > 8) __nanosleep(32);
        }
        (void)ok;
        return;
    }

    const int n_groups = __ldcg(hdr_g + HDR_N_GROUPS);
    const int n_gu = n_groups * tiles_i;

    if (warp == kEpiWarp) {
        // ---- gate_up epilogue: sum the 8 warps' partials in warp order, h = silu(g) * u
        int it = 0;
        for (int item = blockIdx.x; item < n_gu; item += G, ++it) {
            const int rs = it & 1;
            if (!mbar_wait_bounded(&red_full[rs], (it >> 1) & 1)) {
                report_timeout(P);
                break;
            }
            float sg[4] = {0.f, 0.f, 0.f, 0.f}, su[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int w = 0; w < kCW; ++w) {
                const float4* p =
                    reinterpret_cast<const float4*>(red + ((rs * kCW + w) * 32 + lane) * 8);
                const float4 a = p[0], b = p[1];
                sg[0] += a.x, sg[1] += a.y, sg[2] += a.z, sg[3] += a.w;
                su[0] += b.x, su[1] += b.y, su[2] += b.z, su[3] += b.w;
            }
            const int* m = meta + rs * 8;
            const int e0 = m[0], nt = m[1], rt = m[2], gid = m[3];
            const float gglob = __int_as_float(m[4]), uglob = __int_as_float(m[5]);
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_empty[rs]);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int row = (lane >> 2) + ((v >> 1) << 3);
                const int n = 2 * (lane & 3) + (v & 1);
                if (n < nt)
                    h16[(int64_t)(e0 + n) * I + rt * 16 + row] =
                        __float2half_rn(silu(sg[v] * gglob) * (su[v] * uglob));
            }
            __syncwarp();
            if (lane == 0) red_release_gpu_add(done + gid, 1);
        }
        return;
    }

    // ---------------- MMA warps
    const int g = lane >> 2, q = lane & 3;
    bool ok = true;
    {
        if (FL.x_res && n_gu > (int)blockIdx.x && !mbar_wait_bounded(x_full, 0)) {
            report_timeout(P);
            ok = false;
        }
        int it = 0;
        for (int item = blockIdx.x; item < n_gu; item += G, ++it) {
            const int st = it % NGU;
            if (ok && !mbar_wait_bounded(&gu_full[st], (it / NGU) & 1)) {
                report_timeout(P);
                ok = false;
            }
            float accg[kAcc][4] = {}, accu[kAcc][4] = {};
            int mv[6] = {0, 0, 0, 0, 0, 0};
            if (ok) {
                const uint8_t* stg = smem + (size_t)st * FL.stage_gu;
                const int* hdr = reinterpret_cast<const int*>(stg);
                mv[0] = hdr[GD_E0], mv[1] = hdr[GD_NT], mv[2] = hdr[GD_RT], mv[3] = hdr[GD_GID];
                {  // the slot's global scales from the pool itself: a refill between the
                   // grouping and this kernel may have replaced the slot's expert
                    const nvmoe_expert_pool& pl = hdr[GD_POOL] ? P.shared : P.pool;
                    mv[4] = __float_as_int(global_of_early(pl.gate, hdr[GD_SLOT]));
                    mv[5] = __float_as_int(global_of_early(pl.up, hdr[GD_SLOT]));
                }
                const bool has_tok = g < mv[1];
                // B rows: the resident row of the lane's token, or the staged row g
                const uint8_t* xb = FL.x_res ? smem + FL.off_x + (has_tok ? hdr[GD_TOK + g] : 0) * xrow
                                             : stg + og_x + g * xrow;
                const __half* xs = reinterpret_cast<const __half*>(xb);
                if constexpr (TPW > 0) {
#pragma unroll
                    for (int t = 0; t < TPW; ++t)
                        gate_up_tile<Fmt>(stg + kStageHdr, stg + og_uc, stg + og_gs, stg + og_us,
                                          cbg, sbg, aux, xs, has_tok, (warp * TPW + t) * Fmt::kWarpTileK,
                                          g, q, accg, accu);
                } else {
                    const int kw = H / kCW;
                    for (int k0 = warp * kw; k0 < (warp + 1) * kw; k0 += Fmt::kWarpTileK)
                        gate_up_tile<Fmt>(stg + kStageHdr, stg + og_uc, stg + og_gs, stg + og_us,
                                          cbg, sbg, aux, xs, has_tok, k0, g, q, accg, accu);
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&gu_empty[st]);
            fold_acc(accg);
            fold_acc(accu);
            const int rs = it & 1;
            if (ok && !mbar_wait_bounded(&red_empty[rs], ((it >> 1) & 1) ^ 1)) {
                report_timeout(P);
                ok = false;
            }
            float4* rw = reinterpret_cast<float4*>(red + ((rs * kCW + warp) * 32 + lane) * 8);
            rw[0] = make_float4(accg[0][0], accg[0][1], accg[0][2], accg[0][3]);
            rw[1] = make_float4(accu[0][0], accu[0][1], accu[0][2], accu[0][3]);
            if (warp == 0 && lane < 6) {
                // lane i stores field i (selects, not an indexed register array)
                int v = mv[0];
                v = lane == 1 ? mv[1] : v;
                v = lane == 2 ? mv[2] : v;
                v = lane == 3 ? mv[3] : v;
                v = lane == 4 ? mv[4] : v;
                v = lane == 5 ? mv[5] : v;
                meta[rs * 8 + lane] = v;
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&red_full[rs]);
        }
        // this warp reads no gate_up stage any more: the ring may hold down stages
        __syncwarp();
        if (lane == 0) mbar_arrive(gu_drained);
    }

    // ---- down: warp w owns the ring uses j = w, w + 8, ... (one use = one group of a row tile)
    float* ypart = P.ypart_smem ? reinterpret_cast<float*>(smem + FL.off_yp)
                                : wsp<float>(P, P.L.ypart);
    const int ypstride = P.ypart_smem ? 16 : H;  // floats between entries
    const int* ent_of = wsp<int>(P, P.L.ent_of);
    const int K1 = P.top_k + 1;
    int j = 0;
    for (int rt = G - 1 - (int)blockIdx.x; rt < n_dn; rt += G) {
        const int ypcol = P.ypart_smem ? 0 : rt * 16;
        for (int grp = 0; grp < n_groups; ++grp, ++j) {
            // use j of the down ring goes to warp j % 8 and the ring has a multiple of 8 stages,
            // so each stage is always consumed by the same warp, in order: a warp is never a
            // whole phase ahead of a stage's barrier (parity would alias)
            if (j % kCW != warp) continue;
            const int st = j % NDT;
            if (ok && !mbar_wait_bounded(&dn_full[st], (j / NDT) & 1)) {
                report_timeout(P);
                ok = false;
            }
            __syncwarp();
            float acc[kAcc][4] = {};
            int e0 = 0, nt = 0;
            float dglob = 0.f, w_lo = 0.f, w_hi = 0.f;
            if (ok) {  // (the producer released the stage after the group's h was complete and
                       // put the down global scale and, for the shared expert, the gates into it)
                const uint8_t* stg = dn_stage(st);
                const int* hdr = reinterpret_cast<const int*>(stg);
                e0 = hdr[GD_E0], nt = hdr[GD_NT];
                dglob = __int_as_float(hdr[GD_DGLOB]);
                w_lo = __int_as_float(hdr[GD_W + 2 * q]);
                w_hi = __int_as_float(hdr[GD_W + 2 * q + 1]);
                const __half* hrow = g < nt ? h16 + (int64_t)(e0 + g) * I : nullptr;
                if constexpr (TD > 0) {
                    uint4 hb[TD][Fmt::kSteps / 2];
#pragma unroll
                    for (int t = 0; t < TD; ++t)
                        load_h_tile<Fmt>(hrow, t * Fmt::kWarpTileK, q, hb[t]);
#pragma unroll
                    for (int t = 0; t < TD; ++t)
                        down_tile<Fmt>(stg + kStageHdr, stg + od_sc, cbd, sbd, aux, hb[t],
                                       t * Fmt::kWarpTileK, g, q, acc);
                } else {
                    for (int k0 = 0; k0 < I; k0 += Fmt::kWarpTileK) {
                        uint4 hb[Fmt::kSteps / 2];
                        load_h_tile<Fmt>(hrow, k0, q, hb);
                        down_tile<Fmt>(stg + kStageHdr, stg + od_sc, cbd, sbd, aux, hb, k0, g, q,
                                       acc);
                    }
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&dn_empty[st]);
            fold_acc(acc);
            // C fragment: rows g, g+8; entries 2q, 2q+1 of the group
#pragma unroll
            for (int v = 0; v < 4; ++v) {
                const int row = g + ((v >> 1) << 3);
                const int n = 2 * q + (v & 1);
                if (n < nt)
                    ypart[(int64_t)(e0 + n) * ypstride + ypcol + row] =
                        acc[0][v] * dglob * ((v & 1) ? w_hi : w_lo);
            }
        }
        named_bar_sync(1, kConsumers);
        // y rows of this tile: the entries of each token summed in the order j = 0..k-1, shared
        // (no groups: an upstream error or no valid entry, y = 0 without reading the entry map)
        for (int idx = tid; idx < P.n_tok * 16; idx += kConsumers) {
            const int t = idx >> 4, r = idx & 15;
            float sum = 0.f;
            for (int jj = 0; jj < (n_groups > 0 ? K1 : 0); ++jj) {
                const int e = ent_of[t * K1 + jj];
                if (e >= 0) sum += ypart[(int64_t)e * ypstride + ypcol + r];
            }
            P.y[(int64_t)t * P.y_stride + rt * 16 + r] = f32_to_bf16_bits(sum);
        }
        named_bar_sync(1, kConsumers);  // y_part is reused by the next row tile
    }
}

bool pool_ok(const nvmoe_expert_pool& p) {
    return p.gate.data && p.up.data && p.down.data && p.hidden > 0 && p.inter > 0 &&
           p.n_slots > 0;
}

// Rows are staged with 1-D bulk copies (TMA), which need 16-byte aligned addresses and sizes;
// reject any bank whose base or strides would break that alignment.
// Bulk copies move 16 rows at a time: either as one run (rows contiguous) or row by row (each
// row a multiple of 16 bytes); row_bytes is the format's bytes per row of K values.
bool bank_aligned(const nvmoe_matrix_bank& b, bool nvfp4, int row_bytes) {
    const uintptr_t d = reinterpret_cast<uintptr_t>(b.data);
    if ((d & 15) || (b.slot_stride & 15)) return false;
    if (b.row_stride != row_bytes && ((b.row_stride & 15) || (row_bytes & 15))) return false;
    if (nvfp4) {
        const uintptr_t s = reinterpret_cast<uintptr_t>(b.scale);
        if (!b.scale || (s & 15) || (b.scale_slot_stride & 15) || (b.scale_row_stride & 15))
            return false;
    }
    return true;
}

bool pool_aligned(const nvmoe_expert_pool& p) {
    const bool nv = p.quant == NVMOE_Q_NVFP4;
    auto rb = [&](int k) {
        return p.quant == NVMOE_Q_NVFP4 ? k / 2
             : p.quant == NVMOE_Q_BF16  ? FmtBf16::code_bytes(k)
             : p.quant == NVMOE_Q_Q2_K  ? FmtQ2K::code_bytes(k)
                                        : FmtIQ2XXS::code_bytes(k);
    };
    return bank_aligned(p.gate, nv, rb(p.hidden)) && bank_aligned(p.up, nv, rb(p.hidden)) &&
           bank_aligned(p.down, nv, rb(p.inter));
}


template <typename Fmt, int TPW>
auto pick_fused(int td) {
    // the down phase keeps all of a group's h fragments in registers for up to 4 K tiles
    return (td == 2) ? ffn_fused<Fmt, TPW, 2>
         : (td == 4) ? ffn_fused<Fmt, TPW, 4>
                     : ffn_fused<Fmt, TPW, 0>;
}

template <typename Fmt>
int launch_fmt(FfnParams& P, cudaStream_t st) {
    const int H = P.pool.hidden, I = P.pool.inter;
    int dev = 0, sms = 0;
    NVMOE_CUDA_TRY(cudaGetDevice(&dev));
    NVMOE_CUDA_TRY(cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev));
    FusedLayout FL{};
    // all token rows resident in shared memory for decode-sized batches, staged per item above
    FL.x_res = P.n_tok <= kGroupMaxTok ? 1 : 0;
    FL.xt = FL.x_res ? 0 : P.grp_tok;
    const int xrow = H * 2 + kXPad;
    FL.stage_gu = round128(kStageHdr + 32 * Fmt::code_bytes(H) + 32 * Fmt::scale_bytes(H) +
                           FL.xt * xrow);
    FL.stage_dn = round128(kStageHdr + 16 * (Fmt::code_bytes(I) + Fmt::scale_bytes(I)));
    const int x_bytes = FL.x_res ? round128(std::max(1, P.n_tok) * xrow) : 0;
    const int red_bytes = 2 * kCW * 32 * 8 * 4, meta_bytes = 2 * 8 * 4;
    const int bar_bytes = 8 * (2 * 4 + 2 * 64 + 6) + 64;
    const int aux_bytes = round128(Fmt::kAuxBytes);
    const int yp_bytes = round128(P.L.n_ent_max * 16 * 4);
    const int fixed = red_bytes + meta_bytes + bar_bytes + x_bytes + aux_bytes;
    // y_part in shared memory when it leaves room for 2 gate_up and 8 down stages
    P.ypart_smem = (fixed + yp_bytes + 2 * FL.stage_gu + kCW * FL.stage_dn <= kSmemCap) ? 1 : 0;
    const int avail = kSmemCap - fixed - (P.ypart_smem ? yp_bytes : 0);
    // down stage counts are multiples of the 8 MMA warps (see the down phase)
    FL.nst_gu = std::min(4, (avail - kCW * FL.stage_dn) / FL.stage_gu);
    // (one stage only for the widest items, e.g. bf16 rows: loads then do not overlap the math)
    if (FL.nst_gu < 1) return NVMOE_ERR_UNSUPPORTED;
    FL.nst_dn = std::min(32, (avail - FL.nst_gu * FL.stage_gu) / FL.stage_dn) / kCW * kCW;
    if (FL.nst_dn < kCW) return NVMOE_ERR_UNSUPPORTED;
    FL.nst_dn_ext = std::min(32, FL.nst_gu * FL.stage_gu / FL.stage_dn) / kCW * kCW;
    FL.off_x = FL.nst_gu * FL.stage_gu;
    FL.off_dn = FL.off_x + x_bytes;
    FL.off_red = FL.off_dn + FL.nst_dn * FL.stage_dn;
    FL.off_meta = FL.off_red + red_bytes;
    FL.off_yp = FL.off_meta + meta_bytes;
    FL.off_aux = FL.off_yp + (P.ypart_smem ? yp_bytes : 0);
    FL.off_bar = FL.off_aux + aux_bytes;
    FL.total = FL.off_bar + 8 * (2 * FL.nst_gu + 2 * (FL.nst_dn + FL.nst_dn_ext) + 6);
    // compile-time K tiles per MMA warp (gate_up) and per down slab where the shape has an
    // instantiation; other shapes take runtime tile loops
    const int tpw = H / (kCW * Fmt::kWarpTileK), td = I / Fmt::kWarpTileK;
    auto kern = (tpw == 1) ? pick_fused<Fmt, 1>(td)
              : (tpw == 2) ? pick_fused<Fmt, 2>(td)
              : (tpw == 4) ? pick_fused<Fmt, 4>(td)
                           : pick_fused<Fmt, 0>(td);
    NVMOE_CUDA_TRY(
        cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, FL.total));
    // at most one CTA per SM and no more CTAs than SMs: every CTA is resident, so the down
    // phase's waits on other CTAs' gate_up rows always end.  In a decode layer step one SM is
    // left to the next step's front kernel, which then runs while this FFN does.
    const int grid = sms - (P.spare_sm && sms > 1 ? 1 : 0);
    const cudaError_t e =
        launch_pdl(kern, dim3(grid), dim3(kFusedThreads), (size_t)FL.total, st, true, P, FL);
    return cuda_status("ffn_fused launch", e);
}

}  // namespace

bool ffn_fp4_eligible(const FfnParams& P);
int ffn_fp4_launch(const FfnParams& P, cudaStream_t st);

int ffn_setup(const nvmoe_ffn_args* args, FfnParams& P) {
    if (!args || !args->pool || !args->x || !args->slot_ids || !args->weights || !args->y)
        return NVMOE_ERR_INVALID_ARG;
    const nvmoe_expert_pool& pool = *args->pool;
    if (!pool_ok(pool)) return NVMOE_ERR_INVALID_ARG;
    if (args->n_tok < 0 || args->top_k <= 0) return NVMOE_ERR_INVALID_ARG;
    const int H = pool.hidden, I = pool.inter;
    if (args->shared) {
        const nvmoe_expert_pool& sp = *args->shared;
        if (!pool_ok(sp) || sp.quant != pool.quant || sp.hidden != H || sp.inter != I)
            return NVMOE_ERR_INVALID_ARG;
    }
    const bool nv = pool.quant == NVMOE_Q_NVFP4, bf = pool.quant == NVMOE_Q_BF16;
    if (!nv && !bf && pool.quant != NVMOE_Q_Q2_K && pool.quant != NVMOE_Q_IQ2_XXS)
        return NVMOE_ERR_UNSUPPORTED;
    // warp tiling: gate_up K = H over 8 warps, down K = I per warp, 16-row tiles; K tiles of
    // 128 values (NVFP4) or one 256-value super-block (Q2_K / IQ2_XXS)
    // (NVFP4 shapes with H and I multiples of 256 also run on the FP4 tensor-core kernel, which
    // has no further constraint; ffn_fp4_eligible decides below)
    const int tk = nv ? FmtNvfp4::kWarpTileK : bf ? FmtBf16::kWarpTileK : FmtQ2K::kWarpTileK;
    const bool mma_shape = H % (kConsumerWarps * tk) == 0 && I % tk == 0 && I % 16 == 0;
    const bool fp4_shape = nv && H % 256 == 0 && I % 256 == 0;
    if (!mma_shape && !fp4_shape) return NVMOE_ERR_UNSUPPORTED;
    if (nv && (!pool.gate.scale || !pool.up.scale || !pool.down.scale))
        return NVMOE_ERR_INVALID_ARG;
    if (!pool_aligned(pool) || (args->shared && !pool_aligned(*args->shared)))
        return NVMOE_ERR_INVALID_ARG;
    auto row_bytes = [&](int k) {
        return nv ? k / 2 : bf ? FmtBf16::code_bytes(k)
             : pool.quant == NVMOE_Q_Q2_K ? FmtQ2K::code_bytes(k) : FmtIQ2XXS::code_bytes(k);
    };
    const int rbh = row_bytes(H), rbi = row_bytes(I);
    if (pool.gate.row_stride < rbh || pool.up.row_stride < rbh || pool.down.row_stride < rbi)
        return NVMOE_ERR_INVALID_ARG;
    if (nv && (pool.gate.scale_row_stride < H / 16 || pool.down.scale_row_stride < I / 16))
        return NVMOE_ERR_INVALID_ARG;
    const uint32_t* aux_table = nullptr;
    if (pool.quant == NVMOE_Q_IQ2_XXS) {
        int dev = 0;
        NVMOE_CUDA_TRY(cudaGetDevice(&dev));
        if (!iq2xxs_grid_ready(dev)) return NVMOE_ERR_NO_TABLES;
        aux_table = reinterpret_cast<const uint32_t*>(iq2xxs_grid_device_ptr());
        if (!aux_table) return NVMOE_ERR_NO_TABLES;
    }
    if (args->x_row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(args->x) & 15))
        return NVMOE_ERR_INVALID_ARG;
    const WsLayout L = ws_layout(args->n_tok > 0 ? args->n_tok : 1, args->top_k, H, I, pool.n_slots);
    if (!args->workspace || args->workspace_bytes < L.total ||
        (reinterpret_cast<uintptr_t>(args->workspace) & 255))
        return NVMOE_ERR_WORKSPACE;
    P = FfnParams{};
    P.pool = pool;
    P.has_shared = args->shared ? 1 : 0;
    P.shared = args->shared ? *args->shared : pool;
    P.shared_gate = args->shared ? args->shared_gate : nullptr;
    P.x = args->x;
    P.x_stride = args->x_row_stride;
    P.ids = args->slot_ids;
    P.ids_stride = args->ids_row_stride;
    P.w = args->weights;
    P.w_stride = args->weights_row_stride;
    P.top_k = args->top_k;
    P.n_tok = args->n_tok;
    P.y = args->y;
    P.y_stride = args->y_row_stride;
    P.ws = static_cast<unsigned char*>(args->workspace);
    P.L = L;
    P.status = args->status;
    // groups never exceed the token count, so a group's x rows fit the stage even when the
    // caller's slot ids repeat a slot within a token
    P.grp_tok = std::max(1, std::min(kGroupMaxTok, args->n_tok));
    P.aux_table = aux_table;
    if (args->kernel < NVMOE_KERNEL_DEFAULT || args->kernel > NVMOE_KERNEL_F16)
        return NVMOE_ERR_INVALID_ARG;
    P.kernel = args->kernel;
    P.use_fp4 = ffn_fp4_eligible(P) ? 1 : 0;
    if (!P.use_fp4 && !mma_shape) return NVMOE_ERR_UNSUPPORTED;
    return NVMOE_OK;
}

int ffn_launch_main(FfnParams& P, cudaStream_t st) {
    if (P.use_fp4) return ffn_fp4_launch(P, st);
    switch (P.pool.quant) {
        case NVMOE_Q_Q2_K: return launch_fmt<FmtQ2K>(P, st);
        case NVMOE_Q_IQ2_XXS: return launch_fmt<FmtIQ2XXS>(P, st);
        case NVMOE_Q_BF16: return launch_fmt<FmtBf16>(P, st);
        default: return launch_fmt<FmtNvfp4>(P, st);
    }
}

int ffn_launch_prep(FfnParams& P, cudaStream_t st) {
    const size_t prep_smem = (size_t)P.pool.n_slots * 4;
    if (prep_smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
    if (prep_smem > 48 * 1024)
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_prep_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)prep_smem));
    const int conv_blocks = std::min(P.n_tok, 2 * kNumSMs);
    cudaError_t e = launch_pdl(ffn_prep_kernel, dim3(conv_blocks + 1), dim3(kPrepThreads),
                               prep_smem, st, true, P);
    return cuda_status("ffn_prep launch", e);
}

}  // namespace nvmoe

extern "C" size_t nvmoe_moe_ffn_workspace_size(int n_tok, int top_k, int hidden, int inter,
                                               int n_slots) {
    if (n_tok <= 0 || top_k <= 0 || hidden <= 0 || inter <= 0 || n_slots <= 0) return 0;
    return nvmoe::ws_layout(n_tok, top_k, hidden, inter, n_slots).total;
}

extern "C" int nvmoe_moe_ffn_path(const nvmoe_ffn_args* args) {
    nvmoe::FfnParams P;
    const int rc = nvmoe::ffn_setup(args, P);
    if (rc != NVMOE_OK) return rc;
    return P.use_fp4 ? NVMOE_FFN_PATH_FP4 : NVMOE_FFN_PATH_MMA;
}

extern "C" int nvmoe_moe_ffn_prepare(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    FfnParams P;
    const int rc = ffn_setup(args, P);
    if (rc != NVMOE_OK) return rc;
    if (args->n_tok == 0) return NVMOE_OK;
    return ffn_launch_prep(P, (cudaStream_t)stream);
}

extern "C" int nvmoe_moe_ffn_execute(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    FfnParams P;
    const int rc = ffn_setup(args, P);
    if (rc != NVMOE_OK) return rc;
    if (args->n_tok == 0) return NVMOE_OK;
    return ffn_launch_main(P, (cudaStream_t)stream);
}

extern "C" int nvmoe_moe_ffn(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    FfnParams P;
    const int rc = ffn_setup(args, P);
    if (rc != NVMOE_OK) return rc;
    if (args->n_tok == 0) return NVMOE_OK;
    cudaStream_t st = (cudaStream_t)stream;
    const int r1 = ffn_launch_prep(P, st);
    if (r1 != NVMOE_OK) return r1;
    return ffn_launch_main(P, st);
}
