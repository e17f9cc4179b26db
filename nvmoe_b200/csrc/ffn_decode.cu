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
//           items (token group x 16 rows of gate and of up) and then down units (up to 64 rows
//           of H of one group) with 1-D bulk copies (TMA) into two rings of shared-memory
//           stages; 8 MMA warps dequantise A fragments in registers from the staged bytes and
//           run m16n8k16 f16 MMAs (fp32 accumulate); an epilogue warp sums the gate_up partials
//           of the 8 warps and stores h = silu(g) * u (f16); the down producer publishes each
//           finished row tile on a per-group counter; a down unit starts once its group's
//           counter is complete and writes w * down(h) per entry into y_part; after a grid-wide
//           count of finished units every CTA sums its share of y over each token's entries in
//           the fixed order j = 0..k-1, shared, and stores bf16 y.  No atomics on data,
//           deterministic.
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
#pragma unroll 1
        for (int r = 0; r < rows; ++r)
            bulk_g2s_stream(dst + r * row_bytes, src + r * stride, (uint32_t)row_bytes, bar, pol);
    }
}

// ------------------------------------------------------------------ 2. fused gate_up + down
// Shared memory: [gate_up ring][resident x][down ring][red: 2 x 8 warps x 32 lanes x 8
// floats][meta: 2 x 8 ints, publication ring][mbarriers].  Once the gate_up phase has drained,
// its ring's bytes hold further down stages.
//   gate_up stage: [record 128 B] gate codes [16][H/2] | up codes | gate scales [16][H/16] |
//                  up scales | x [XT][H + 8] f16 when x is staged per item (XT = the largest
//                  group of this launch; the 8 extra halves per row only spread the rows over
//                  the banks); resident x: [n_tok][H + 8] f16 once per CTA (n_tok <= 8)
//   down stage   : [record 128 B] codes [dn_rows][I/2] | scales [dn_rows][I/16]
struct FusedLayout {
    int stage_gu, stage_dn;  // bytes per stage
    int nst_gu;              // gate_up ring stages
    int nst_dn;              // down stages in their own region (a multiple of the warp groups)
    int nst_dn_ext;          // down stages carved from the gate_up ring once it has drained
    int dn_rows;             // rows of H per down unit (64, 32 or 16: 16 per MMA warp)
    int xt;                  // x rows per gate_up stage (staged x), 0 with resident x
    int x_res;               // 1: every token row resident in shared memory, loaded once
    int off_x, off_dn, off_red, off_meta, off_bar, total;
    int off_aux;             // the format's lookup table (IQ2_XXS grid)
};

__host__ __device__ inline int round128(int v) { return (v + 127) / 128 * 128; }

// One 128-wide K tile of a 16-row gate + up item: rows g and g + 8 of both matrices for the
// lane quarter q, B = the activations of the group's tokens (token g of the lane).  Lanes past
// the group's tokens load some valid row: their output columns are never stored, and loads
// without a condition keep the tile straight-line code.
// The MMAs of consecutive steps go to kAcc independent accumulators (a single accumulator
// chains every mma.sync on the previous one's result and leaves the warp latency-bound); the
// accumulators are summed in a fixed order at the end of the item.
constexpr int kAcc = 8;
// entries per token (top-k + the shared expert) whose partials the final sum loads at once
constexpr int kSumK = 12;

template <typename Fmt>
__device__ __forceinline__ void gate_up_tile(const uint8_t* gcode, const uint8_t* ucode,
                                             const uint8_t* gsc, const uint8_t* usc, int cb,
                                             int sb, const uint32_t* aux, const __half* xs,
                                             int k0,
                                             int g, int q, float (&accg)[kAcc][4],
                                             float (&accu)[kAcc][4]) {
    typename Fmt::Row ga, gb, ua, ub;
    Fmt::load_smem(ga, gcode + g * cb, gsc + g * sb, k0, q, aux);
    Fmt::load_smem(gb, gcode + (g + 8) * cb, gsc + (g + 8) * sb, k0, q, aux);
    Fmt::load_smem(ua, ucode + g * cb, usc + g * sb, k0, q, aux);
    Fmt::load_smem(ub, ucode + (g + 8) * cb, usc + (g + 8) * sb, k0, q, aux);
#pragma unroll
    for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
        const uint4 xb = *reinterpret_cast<const uint4*>(xs + k0 + Fmt::kofs(q, s2));
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

// h fragments of one K tile for token row hrow, in the order of the format's step pairs, read
// through L2 (h is written by other CTAs of this grid).
template <typename Fmt>
__device__ __forceinline__ void load_h_tile(const __half* hrow, int k0, int q,
                                            uint4 (&hb)[Fmt::kSteps / 2]) {
#pragma unroll
    for (int i = 0; i < Fmt::kSteps / 2; ++i)
        hb[i] = __ldcg(reinterpret_cast<const uint4*>(hrow + k0 + Fmt::kofs(q, 2 * i)));
}

__device__ __forceinline__ int ld_relaxed_gpu(const int* p) {
    int v;
    asm volatile("ld.relaxed.gpu.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void fence_acq_rel_gpu() {
    asm volatile("fence.acq_rel.gpu;" ::: "memory");
}
__device__ __forceinline__ void red_relaxed_gpu_add(int* p, int v) {
    asm volatile("red.relaxed.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_release_cta(int* p, int v) {
    asm volatile("st.release.cta.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(p)), "r"(v) : "memory");
}
__device__ __forceinline__ int ld_acquire_cta(const int* p) {
    int v;
    asm volatile("ld.acquire.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}
__device__ __forceinline__ int ld_relaxed_cta(const int* p) {
    int v;
    asm volatile("ld.relaxed.cta.shared::cta.b32 %0, [%1];" : "=r"(v) : "r"(smem_u32(p)) : "memory");
    return v;
}

// Publication of finished h row tiles.  The epilogue warp stores a gate_up item's h rows and
// hands the item's group to the down producer warp through a ring in shared memory (release /
// acquire at CTA scope); the down producer publishes everything handed over so far with one
// gpu-scope fence and one relaxed count per item.  The fence waits until the stores have
// reached L2 (about a microsecond under the weight stream), so it runs on the warp that is not
// on the gate_up critical path, and it covers every item stored meanwhile.
//   pub[0] items handed over, pub[1] items published, pub[2] items the epilogue finished with
//   (-1 while it runs), pub[4 + i % kPubRing] the group of item i
constexpr int kPubRing = 32;
constexpr int kPubInts = 4 + kPubRing;

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
constexpr int kCW = kConsumerWarps;       // MMA warps
// Hardware warp of each role: the 8 MMA warps are warps 0-7 (index mw = warp), then the
// control warps.
constexpr int kProdGU = kCW;              // bulk-copy producer of the gate_up items
constexpr int kEpiWarp = kCW + 1;         // gate/up cross-warp sum + SwiGLU + h store
constexpr int kProdDN = kCW + 2;          // bulk-copy producer of the down units; publisher
constexpr int kRefillWarp = kCW + 3;      // copies this call's misses in from the host tier
constexpr int kFusedThreads = (kCW + 4) * 32;

// Persistent expert FFN, one CTA per SM.  CTA c runs
//   gate_up items c, c + G, ... (item = token group x 16 rows of gate and of up, full K = H),
//   then down units c, c + G, ... (unit = dn_rows rows of H of one group, K = I), numbered
//   group-major so that the groups whose h completes first come first, then its share of y.
// Roles: two producer warps stream the two phases' weights into their rings (down weights do
// not depend on h, so they are in flight while gate_up runs); the 8 MMA warps split K of a
// gate_up item (TPW tiles each, straight-line code) and hand their partial sums to the
// epilogue warp through a 2-deep ring, so they never wait for the cross-warp sum; the epilogue
// warp stores h and hands the item to the down producer warp, which counts the group's
// finished row tiles (fence, then relaxed counts); a down MMA warp owns whole groups and starts
// a group once its count is complete (acquire).
template <typename Fmt, int TPW, int TD>
__global__ void __launch_bounds__(kFusedThreads, 1) ffn_fused(FfnParams P, FusedLayout FL) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // With compile-time K tiles (TPW, TD > 0) the host has checked H = TPW x 8 warps x tile and
    // I = TD x tile, so H, I and every row stride and offset inside a stage are constants: the
    // tile loops then address shared memory with immediate offsets (runtime strides measured
    // almost twice as slow in the gate_up tile).
    const int H = TPW > 0 ? TPW * kCW * Fmt::kWarpTileK : P.pool.hidden;
    const int I = TD > 0 ? TD * Fmt::kWarpTileK : P.pool.inter;
    const int G = gridDim.x;
    // (the down producer gives each ring stage to one lane: at most 32 stages are used)
    const int NGU = FL.nst_gu, NDT = FL.nst_dn + FL.nst_dn_ext;
    // down units: dn_rows rows of H of one group; its dn_rows / 16 MMA warps form a warp group
    const int dn_rows = FL.dn_rows, wpu = dn_rows / 16, n_wg = kCW / wpu;
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
    int* pub = meta + 16;
    if (tid == 0) {
        pub[0] = 0, pub[1] = 0, pub[2] = -1;
        for (int s = 0; s < NGU; ++s) mbar_init(&gu_full[s], 1), mbar_init(&gu_empty[s], kCW);
        for (int s = 0; s < NDT; ++s) mbar_init(&dn_full[s], 1), mbar_init(&dn_empty[s], wpu);
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

    const int tiles_i = I / 16, nb = H / dn_rows;
    const int cbg = Fmt::code_bytes(H), sbg = Fmt::scale_bytes(H);
    const int cbd = Fmt::code_bytes(I), sbd = Fmt::scale_bytes(I);
    const int og_uc = kStageHdr + 16 * cbg, og_gs = kStageHdr + 32 * cbg;
    const int og_us = og_gs + 16 * sbg, og_x = og_us + 16 * sbg;
    const int od_sc = kStageHdr + dn_rows * cbd;
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
#pragma unroll 1
            for (int t = 0; t < P.n_tok; ++t)
                bulk_g2s(smem + FL.off_x + t * xrow, x16 + (int64_t)t * H, (uint32_t)(H * 2), x_full);
        }
        bool ok = true;
        int it = 0;
#pragma unroll 1
        for (int base = blockIdx.x; base < n_gu && ok; base += 32 * G) {
            const int mine = base + lane * G;
            if (base != (int)blockIdx.x && mine < n_gu) load_record(P, mine / tiles_i, rec);
            const int n_here = min(32, (n_gu - base + G - 1) / G);
            // Lane i holds item i's record and issues it (no shuffles of the record); the loop
            // is not unrolled, so every item runs the same short stretch of code, which stays in
            // the instruction cache (unrolled copies were cold on every item, and their fetches,
            // not the weight stream, paced the gate_up phase).
#pragma unroll 1
            for (int i = 0; i < n_here; ++i, ++it) {
                if (lane == i) {
                    const int* rv = reinterpret_cast<const int*>(rec);
                    const int item = mine;
                    const int st = it % NGU;
                    if (!mbar_wait_bounded(&gu_empty[st], ((it / NGU) & 1) ^ 1)) {
                        report_timeout(P);
                        ok = false;
                    } else {
                        uint8_t* stg = smem + (size_t)st * FL.stage_gu;
                        int* hdr = reinterpret_cast<int*>(stg);
                        copy_record(hdr, rec);
                        const int miss = rv[GD_MISS];
                        if (miss > 0 && !refill_wait(P, miss - 1, 0)) {
                            report_timeout(P);
                            ok = false;
                        }
                        const int rt = item % tiles_i;
                        hdr[GD_RT] = rt;
                        hdr[GD_GID] = item / tiles_i;
                        const int sh = rv[GD_POOL];
                        const BankSel bg = bank_sel(sh, P.pool.gate, P.shared.gate);
                        const BankSel bu = bank_sel(sh, P.pool.up, P.shared.up);
                        const int slot = rv[GD_SLOT], nt = rv[GD_NT];
                        const int64_t r0 = (int64_t)rt * 16;
                        mbar_arrive_expect_tx(
                            &gu_full[st],
                            (uint32_t)(32 * cbg + 32 * sbg + (FL.x_res ? 0 : nt * H * 2)));
                        bulk_rows(stg + kStageHdr,
                                  bg.data + slot * bg.slot_stride + r0 * bg.row_stride, 16, cbg,
                                  bg.row_stride, &gu_full[st]);
                        bulk_rows(stg + og_uc,
                                  bu.data + slot * bu.slot_stride + r0 * bu.row_stride, 16, cbg,
                                  bu.row_stride, &gu_full[st]);
                        if (sbg > 0) {  // formats with a separate scale bank
                            bulk_rows(stg + og_gs,
                                      bg.scale + slot * bg.scale_slot_stride +
                                          r0 * bg.scale_row_stride,
                                      16, sbg, bg.scale_row_stride, &gu_full[st]);
                            bulk_rows(stg + og_us,
                                      bu.scale + slot * bu.scale_slot_stride +
                                          r0 * bu.scale_row_stride,
                                      16, sbg, bu.scale_row_stride, &gu_full[st]);
                        }
                        if (!FL.x_res)
#pragma unroll 1
                            for (int n = 0; n < nt; ++n)
                                bulk_g2s(stg + og_x + n * xrow, x16 + (int64_t)hdr[GD_TOK + n] * H,
                                         (uint32_t)(H * 2), &gu_full[st]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, i);
                if (!ok) break;
            }
        }
        return;
    }

    if (warp == kProdDN) {
        // down units: unit j of this CTA is u = blockIdx.x + j G (group u / nb, rows
        // [dn_rows (u % nb), + dn_rows) of H) in stage j % NDT.  Lane i owns stage i and runs its
        // units i, i + NDT, ... as a state machine of its own, polled without blocking (a lane
        // that waited in a loop of its own would hold the others back):
        //   the gate_up ring drained (stages in its bytes) -> stage free -> missed slot's banks
        //   in -> rows requested (expect_tx, bulk copies) -> the group's h complete: down global
        //   scale and shared-expert gates into the stage's record copy, arrive (the MMA warp
        //   reads h without an acquire of its own: release -> acquire here, then the barrier)
        enum { S_DRAIN, S_FREE, S_REFILL, S_ISSUE, S_H, S_DONE };
        const int n_groups = __ldcg(hdr_g + HDR_N_GROUPS);
        const float* sgate = (P.has_shared && P.shared_gate) ? wsp<float>(P, P.L.sg) : nullptr;
        const int n_units = n_groups * nb;
        const int total = (int)blockIdx.x < n_units ? (n_units - 1 - (int)blockIdx.x) / G + 1 : 0;
        auto group_of = [&](int jj) { return ((int)blockIdx.x + jj * G) / nb; };
        int j = lane;
        int state = (lane >= NDT || j >= total) ? S_DONE : (lane >= FL.nst_dn ? S_DRAIN : S_FREE);
        uint8_t* stg = dn_stage(lane < NDT ? lane : 0);
        int* hdr = reinterpret_cast<int*>(stg);
        int4 r[kDescInts / 4];
        if (state != S_DONE) load_record(P, group_of(j), r);
        float dgl = 1.f;
        bool ok = true;
        unsigned backoff = 32;
        int published = 0;
        bool pub_open = lane == 0;  // lane 0 publishes the epilogue's items until it finishes
        for (uint32_t w = 0; __any_sync(0xffffffffu, state != S_DONE || pub_open); ++w) {
            if (w == (1u << 24)) {  // a few seconds: give up
                if (state != S_DONE || pub_open) {
                    report_timeout(P);
                    ok = false;
                }
                break;
            }
            const int state0 = state;
            bool moved = false;
            if (pub_open) {
                const int fin = ld_acquire_cta(pub + 2);  // (read before the count)
                const int handed = ld_acquire_cta(pub);
                if (handed > published) {
                    fence_acq_rel_gpu();
#pragma unroll 1
                    for (int i = published; i < handed; ++i)
                        red_relaxed_gpu_add(done + pub[4 + i % kPubRing], 1);
                    published = handed;
                    st_release_cta(pub + 1, published);
                    moved = true;
                }
                if (fin >= 0 && published >= fin) pub_open = false;
            }
            if (state == S_DRAIN && mbar_test_wait(gu_drained, 0)) state = S_FREE;
            if (state == S_FREE && mbar_test_wait(&dn_empty[lane], ((j / NDT) & 1) ^ 1)) {
                copy_record(hdr, r);
                hdr[GD_GID] = group_of(j);
                state = hdr[GD_MISS] > 0 ? S_REFILL : S_ISSUE;
            }
            if (state == S_REFILL && refill_ready(P, hdr[GD_MISS] - 1, 1)) state = S_ISSUE;
            if (state == S_ISSUE) {
                const BankSel bd = bank_sel(hdr[GD_POOL], P.pool.down, P.shared.down);
                const int slot = hdr[GD_SLOT];
                const int64_t r0 = (int64_t)(((int)blockIdx.x + j * G) % nb) * dn_rows;
                dgl = global_of_sel(bd, slot);
                mbar_expect_tx(&dn_full[lane], (uint32_t)(dn_rows * (cbd + sbd)));
                bulk_rows(stg + kStageHdr, bd.data + slot * bd.slot_stride + r0 * bd.row_stride,
                          dn_rows, cbd, bd.row_stride, &dn_full[lane]);
                if (sbd > 0)
                    bulk_rows(stg + od_sc,
                              bd.scale + slot * bd.scale_slot_stride + r0 * bd.scale_row_stride,
                              dn_rows, sbd, bd.scale_row_stride, &dn_full[lane]);
                state = S_H;
            }
            // (relaxed polls; the acquire is one fence once the count is complete)
            if (state == S_H && ld_relaxed_gpu(done + group_of(j)) >= tiles_i) {
                fence_acq_rel_gpu();
                hdr[GD_DGLOB] = __float_as_int(dgl);
                if (hdr[GD_POOL] && sgate) {
                    const int nt = hdr[GD_NT];
#pragma unroll 1
                    for (int k = 0; k < nt; ++k)
                        hdr[GD_W + k] = __float_as_int(__ldcg(sgate + hdr[GD_TOK + k]));
                }
                mbar_arrive(&dn_full[lane]);
                j += NDT;
                state = S_DONE;
                if (j < total) {
                    load_record(P, group_of(j), r);  // (used once the stage is free again)
                    state = S_FREE;
                }
            }
            // back off while no lane moves (most of the gate_up phase: every lane waits for h)
            if (__any_sync(0xffffffffu, state != state0 || moved)) {
                backoff = 32;
            } else if (w > 8) {
                __nanosleep(backoff);
                backoff = min(2 * backoff, 256);
            }
        }
        (void)ok;
        return;
    }

    const int n_groups = __ldcg(hdr_g + HDR_N_GROUPS);
    const int n_gu = n_groups * tiles_i;

    if (warp == kEpiWarp) {
        // ---- gate_up epilogue: sum the 8 warps' partials in warp order, h = silu(g) * u, then
        // hand the item to the down producer for publication
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
            int ring_ok = 1;
            if (lane == 0) {
                // a free ring entry: the publisher is less than kPubRing items behind
                for (uint32_t i = 0; it - ld_relaxed_cta(pub + 1) >= kPubRing; ++i) {
                    if (i == (1u << 22)) {
                        report_timeout(P);
                        ring_ok = 0;
                        break;
                    }
                    __nanosleep(64);
                }
                if (ring_ok) {
                    pub[4 + it % kPubRing] = gid;
                    st_release_cta(pub, it + 1);  // (orders the warp's h stores before it)
                }
            }
            if (!__shfl_sync(0xffffffffu, ring_ok, 0)) break;
        }
        if (lane == 0) st_release_cta(pub + 2, it);
        return;
    }

    // ---------------- MMA warps (mw = 0..7, ctid = this thread's index among the MMA threads)
    const int mw = warp, ctid = tid;
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
                if (mw == 0) {  // (only warp 0 hands them on) the slot's global scales from
                                // the pool itself: a refill between the grouping and this
                                // kernel may have replaced the slot's expert
                    const int sh = hdr[GD_POOL], slot = hdr[GD_SLOT];
                    mv[4] = __float_as_int(global_of_sel(bank_sel(sh, P.pool.gate, P.shared.gate), slot));
                    mv[5] = __float_as_int(global_of_sel(bank_sel(sh, P.pool.up, P.shared.up), slot));
                }
                const bool has_tok = g < mv[1];
                // B rows: the resident row of the lane's token, or the staged row g (lanes
                // without a token: the row of the group's first token)
                const uint8_t* xb = FL.x_res ? smem + FL.off_x + hdr[GD_TOK + (has_tok ? g : 0)] * xrow
                                             : stg + og_x + (has_tok ? g : 0) * xrow;
                const __half* xs = reinterpret_cast<const __half*>(xb);
                if constexpr (TPW > 0) {
                    // (one tile body: the warp's K tiles run through the same code)
#pragma unroll 1
                    for (int t = 0; t < TPW; ++t)
                        gate_up_tile<Fmt>(stg + kStageHdr, stg + og_uc, stg + og_gs, stg + og_us,
                                          cbg, sbg, aux, xs, (mw * TPW + t) * Fmt::kWarpTileK,
                                          g, q, accg, accu);
                } else {
                    const int kw = H / kCW;
                    for (int k0 = mw * kw; k0 < (mw + 1) * kw; k0 += Fmt::kWarpTileK)
                        gate_up_tile<Fmt>(stg + kStageHdr, stg + og_uc, stg + og_gs, stg + og_us,
                                          cbg, sbg, aux, xs, k0, g, q, accg, accu);
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
            float4* rw = reinterpret_cast<float4*>(red + ((rs * kCW + mw) * 32 + lane) * 8);
            rw[0] = make_float4(accg[0][0], accg[0][1], accg[0][2], accg[0][3]);
            rw[1] = make_float4(accu[0][0], accu[0][1], accu[0][2], accu[0][3]);
            if (mw == 0 && lane < 6) {
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

    // ---- down: unit j of this CTA (u = blockIdx.x + j G: group u / nb, rows [dn_rows (u % nb),
    // + dn_rows) of H) goes to warp group j % n_wg, whose warp wsl takes the unit's rows
    // [16 wsl, 16 wsl + 16).  The ring has a multiple of n_wg stages, so each stage is always
    // consumed by the same warp group, in order: a warp is never a whole phase ahead of a
    // stage's barrier (parity would alias).  Each entry's rows go to y_part [entry][H] (fp32).
    float* ypart = wsp<float>(P, P.L.ypart);
    const int* ent_of = wsp<int>(P, P.L.ent_of);
    const int K1 = P.top_k + 1;
    const int wgi = mw / wpu, wsl = mw % wpu;
    const int n_units = n_groups * nb;
    const int n_local = (int)blockIdx.x < n_units ? (n_units - 1 - (int)blockIdx.x) / G + 1 : 0;
    for (int j = wgi; j < n_local; j += n_wg) {
        const int st = j % NDT;
        if (ok && !mbar_wait_bounded(&dn_full[st], (j / NDT) & 1)) {
            report_timeout(P);
            ok = false;
        }
        __syncwarp();
        float acc[kAcc][4] = {};
        int e0 = 0, nt = 0;
        float dglob = 0.f, w_lo = 0.f, w_hi = 0.f;
        if (ok) {  // (the producer released the stage after the group's h was complete and put
                   // the down global scale and, for the shared expert, the gates into it)
            const uint8_t* stg = dn_stage(st);
            const int* hdr = reinterpret_cast<const int*>(stg);
            e0 = hdr[GD_E0], nt = hdr[GD_NT];
            dglob = __int_as_float(hdr[GD_DGLOB]);
            w_lo = __int_as_float(hdr[GD_W + 2 * q]);
            w_hi = __int_as_float(hdr[GD_W + 2 * q + 1]);
            const uint8_t* code = stg + kStageHdr + wsl * 16 * cbd;
            const uint8_t* sc = stg + od_sc + wsl * 16 * sbd;
            // (lanes past the group's entries read entry 0's row; their columns are not stored)
            const __half* hrow = h16 + (int64_t)(e0 + (g < nt ? g : 0)) * I;
            if constexpr (TD > 0) {
                uint4 hb[TD][Fmt::kSteps / 2];
#pragma unroll
                for (int t = 0; t < TD; ++t) load_h_tile<Fmt>(hrow, t * Fmt::kWarpTileK, q, hb[t]);
#pragma unroll
                for (int t = 0; t < TD; ++t)
                    down_tile<Fmt>(code, sc, cbd, sbd, aux, hb[t], t * Fmt::kWarpTileK, g, q, acc);
            } else {
                for (int k0 = 0; k0 < I; k0 += Fmt::kWarpTileK) {
                    uint4 hb[Fmt::kSteps / 2];
                    load_h_tile<Fmt>(hrow, k0, q, hb);
                    down_tile<Fmt>(code, sc, cbd, sbd, aux, hb, k0, g, q, acc);
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&dn_empty[st]);
        fold_acc(acc);
        // C fragment: rows g, g+8; entries 2q, 2q+1 of the group
        const int row0 = (((int)blockIdx.x + j * G) % nb) * dn_rows + wsl * 16;
#pragma unroll
        for (int v = 0; v < 4; ++v) {
            const int row = g + ((v >> 1) << 3);
            const int n = 2 * q + (v & 1);
            if (n < nt)
                ypart[(int64_t)(e0 + n) * H + row0 + row] =
                    acc[0][v] * dglob * ((v & 1) ? w_hi : w_lo);
        }
    }
    // every unit of the grid done (a count over all CTAs; the grid is resident, one CTA per SM):
    // this CTA's y_part stores, then its count (fence, relaxed add); wait for the total
    named_bar_sync(1, kConsumers);
    int* dn_done = wsp<int>(P, P.L.phase);  // (reset by the grouping before this kernel)
    if (ctid == 0) {
        fence_acq_rel_gpu();
        red_relaxed_gpu_add(dn_done, n_local);
        bool fin = false;
        for (uint32_t i = 0; i < (1u << 22); ++i) {
            if (ld_relaxed_gpu(dn_done) >= n_units) {
                fin = true;
                break;
            }
            __nanosleep(i < 64 ? 32 : 256);
        }
        if (!fin) report_timeout(P);
        fence_acq_rel_gpu();
    }
    named_bar_sync(1, kConsumers);
    // y: this CTA's share of the (token, row) outputs, each token's entries summed in the order
    // j = 0..k-1, shared (no groups: an upstream error or no valid entry, y = 0 without reading
    // the entry map)
    const int n_out = P.n_tok * H;
    const int k1 = n_groups > 0 ? K1 : 0;
    for (int idx = (int)blockIdx.x * kConsumers + ctid; idx < n_out; idx += G * kConsumers) {
        const int t = idx / H, r = idx - t * H;
        float sum = 0.f;
        if (k1 <= kSumK) {
            // every entry index first, then every partial: two round trips to L2 in all, not
            // two per entry (dependent pairs made the slowest CTAs' sums the kernel's tail)
            int e[kSumK];
            float v[kSumK];
#pragma unroll
            for (int jj = 0; jj < kSumK; ++jj) e[jj] = jj < k1 ? __ldg(ent_of + t * K1 + jj) : -1;
#pragma unroll
            for (int jj = 0; jj < kSumK; ++jj)
                v[jj] = e[jj] >= 0 ? __ldcg(ypart + (int64_t)e[jj] * H + r) : 0.f;
#pragma unroll
            for (int jj = 0; jj < kSumK; ++jj)
                if (e[jj] >= 0) sum += v[jj];
        } else {
            for (int jj = 0; jj < k1; ++jj) {
                const int e = __ldg(ent_of + t * K1 + jj);
                if (e >= 0) sum += __ldcg(ypart + (int64_t)e * H + r);
            }
        }
        P.y[(int64_t)t * P.y_stride + r] = f32_to_bf16_bits(sum);
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
    // down units of 64, 32 or 16 rows of H (16 per MMA warp): the largest whose stage stays
    // within 20 KB.  Fewer, larger bulk copies: every copy costs the single-lane producer a
    // fixed issue time, and 16-row units made the down phase issue-bound (2 copies per 4.6 KB).
    const int row_dn = Fmt::code_bytes(I) + Fmt::scale_bytes(I);
    FL.dn_rows = 64;
    while (FL.dn_rows > 16 && kStageHdr + FL.dn_rows * row_dn > 20 * 1024) FL.dn_rows /= 2;
    if (H % FL.dn_rows) return NVMOE_ERR_UNSUPPORTED;
    const int n_wg = kCW / (FL.dn_rows / 16);  // warp groups; down stage counts are multiples
    FL.stage_dn = round128(kStageHdr + FL.dn_rows * row_dn);
    const int x_bytes = FL.x_res ? round128(std::max(1, P.n_tok) * xrow) : 0;
    const int red_bytes = 2 * kCW * 32 * 8 * 4, meta_bytes = round128((16 + kPubInts) * 4);
    const int bar_bytes = 8 * (2 * 4 + 2 * 64 + 6) + 64;
    const int aux_bytes = round128(Fmt::kAuxBytes);
    const int fixed = red_bytes + meta_bytes + bar_bytes + x_bytes + aux_bytes;
    const int avail = kSmemCap - fixed;
    FL.nst_gu = std::min(4, (avail - n_wg * FL.stage_dn) / FL.stage_gu);
    // (one stage only for the widest items, e.g. bf16 rows: loads then do not overlap the math)
    if (FL.nst_gu < 1) return NVMOE_ERR_UNSUPPORTED;
    FL.nst_dn = std::min(32, (avail - FL.nst_gu * FL.stage_gu) / FL.stage_dn) / n_wg * n_wg;
    if (FL.nst_dn < n_wg) return NVMOE_ERR_UNSUPPORTED;
    FL.nst_dn_ext =
        std::min(32 - FL.nst_dn, FL.nst_gu * FL.stage_gu / FL.stage_dn) / n_wg * n_wg;
    FL.off_x = FL.nst_gu * FL.stage_gu;
    FL.off_dn = FL.off_x + x_bytes;
    FL.off_red = FL.off_dn + FL.nst_dn * FL.stage_dn;
    FL.off_meta = FL.off_red + red_bytes;
    FL.off_aux = FL.off_meta + meta_bytes;
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
