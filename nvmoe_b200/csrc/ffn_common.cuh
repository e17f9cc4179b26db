// Shared definitions of the expert-FFN kernels: workspace layout, kernel parameters, token
// groups and the grouping step (shared by the FFN prep kernel and the fused decode front kernel).
#pragma once

#include <string.h>

#include "common.cuh"

namespace nvmoe {

constexpr int kPrepThreads = 256;
constexpr int kGroupMaxTok = 8;  // largest token group (entries), = the MMA N of one tile
constexpr int kDescInts = 32;    // ints per group record (128 bytes)

// Group record: one token group (<= 8 entries of one active slot), complete enough that the FFN
// kernel's producer reads nothing else before it issues the group's weight copies.
enum {
    GD_SLOT = 0,    // slot in its pool
    GD_POOL = 1,    // 0 routed pool, 1 shared expert
    GD_E0 = 2,      // first entry (entries of a group are consecutive)
    GD_NT = 3,      // number of entries
    GD_TOK = 4,     // token of each entry (8)
    GD_RT = 12,     // (stage copies only) row tile of the work item
    GD_GID = 13,    // (stage copies only) group index
    GD_MISS = 14,   // miss index + 1 when this FFN call refills the slot's expert, else 0
    GD_GGLOB = 16,  // unused (the FFN reads the slot's global scales from the pool when it
    GD_UGLOB = 17,  //   runs, after any refill of the slot; the grouping may run before it)
    GD_DGLOB = 18,
    GD_W = 20,      // float: router weight of each entry (8); 1 for the shared expert
};

// ------------------------------------------------------------------ workspace layout
// Tensor-core (block-scaled FP4) FFN path: per-group activation images and counters.
constexpr int kFp4Terms = 4;          // NVFP4 terms per activation (x = sum of 4 scaled E2M1 tiles)
constexpr int kFp4BRows = 4 * 8;      // B rows of a group: kFp4Terms x up to 8 tokens
constexpr int kFp4ImgStage = kFp4BRows * 144;  // one 256-wide K stage: codes rows x 128 B, SF x 16 B
constexpr int kFp4MaxCtas = 160;

struct WsLayout {
    size_t hdr, active_slot, tok_cnt, grp_desc, grp_done, ent_tok, ent_w, ent_of, x16, sg, h16,
        ypart, bimg, ximg, xk, hk, h32, gcnt, phase, rdy, total;
    int a_max, n_ent_max, g_max;
    int jb, rb, ks_gu, ks_dn;  // FP4 path: 64-row j-blocks, 128-row H blocks, K stages (0: off)
};

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline WsLayout ws_layout(int n_tok, int top_k, int H, int I, int n_slots) {
    WsLayout L;
    const int n_route = n_tok * top_k;
    L.a_max = (n_route < n_slots ? n_route : n_slots) + 1;
    L.n_ent_max = n_route + n_tok;
    // a group holds at least one entry; slot s with c_s entries makes ceil(c_s / gt) groups
    const int gt = n_tok < 8 ? (n_tok > 0 ? n_tok : 1) : 8;
    const int g_bound = n_route / gt + L.a_max + (n_tok + gt - 1) / gt + 2;
    L.g_max = L.n_ent_max < g_bound ? L.n_ent_max : g_bound;
    const bool fp4 = H % 256 == 0 && I % 256 == 0;
    L.jb = fp4 ? I / 64 : 0;
    L.rb = fp4 ? H / 128 : 0;
    L.ks_gu = fp4 ? H / 256 : 0;
    L.ks_dn = fp4 ? I / 256 : 0;
    size_t o = 0;
    L.hdr = o;
    o = align_up(o + 64, 256);
    L.active_slot = o;
    o = align_up(o + 4 * (size_t)L.a_max, 256);
    L.tok_cnt = o;
    o = align_up(o + 4 * (size_t)L.a_max, 256);
    L.grp_desc = o;
    o = align_up(o + 4 * (size_t)kDescInts * L.g_max, 256);
    L.grp_done = o;  // per group: gate/up row tiles whose h rows are stored
    o = align_up(o + 4 * (size_t)L.g_max, 256);
    L.ent_tok = o;
    o = align_up(o + 4 * (size_t)L.n_ent_max, 256);
    L.ent_w = o;
    o = align_up(o + 4 * (size_t)L.n_ent_max, 256);
    L.ent_of = o;
    o = align_up(o + 4 * (size_t)L.n_ent_max, 256);
    L.x16 = o;
    o = align_up(o + 2 * (size_t)n_tok * H, 256);
    L.sg = o;
    o = align_up(o + 4 * (size_t)n_tok, 256);
    L.h16 = o;
    o = align_up(o + 2 * (size_t)L.n_ent_max * I, 256);
    L.ypart = o;  // used by the down phase only when its shared-memory copy does not fit
    o = align_up(o + 4 * (size_t)L.n_ent_max * H, 256);
    L.bimg = o;  // per group: the down K stages of the B operand image (h)
    o = align_up(o + (size_t)L.g_max * L.ks_dn * kFp4ImgStage, 1024);
    L.ximg = o;  // per token: gate_up operand rows (2 swizzle phases x K stages x 4 rows x 128 B,
                 // then K stages x 4 rows x 16 B of scales)
    o = align_up(o + (size_t)n_tok * L.ks_gu * (2 * 512 + 64), 1024);
    L.xk = o;  // per token: the power-of-two exponent of its activation terms
    o = align_up(o + 4 * (size_t)n_tok, 256);
    L.hk = o;  // per (group, token of the group): the exponent of its h terms
    o = align_up(o + 4 * (size_t)L.g_max * kGroupMaxTok, 256);
    L.h32 = o;  // per (group, token of the group): h in fp32 [I]
    o = align_up(o + (fp4 ? 4 * (size_t)L.g_max * kGroupMaxTok * I : 0), 256);
    L.gcnt = o;  // per group: gate_up units stored, h rows built
    o = align_up(o + 8 * (size_t)L.g_max, 256);
    L.phase = o;  // grid phase counters of the FP4 kernel (4 ints)
    o = align_up(o + 16, 256);
    L.rdy = o;  // per miss refilled by the FFN: pieces copied of its gate/up and down banks
    o = align_up(o + 8 * (size_t)L.a_max, 256);
    L.total = o;
    return L;
}

enum { HDR_N_ACTIVE = 0, HDR_N_ENT = 1, HDR_STATUS = 2, HDR_N_GROUPS = 3 };

// Misses the FFN kernel copies in from the pinned host tier itself (decode layer step), so the
// copies overlap the hit groups: rows of each bank of each miss in pieces of kRefillPiece bytes.
constexpr int kRefillMaxBanks = 8;
constexpr int kRefillPiece = 8192;
struct FfnRefill {
    nvmoe_refill_bank banks[kRefillMaxBanks];
    int pbase[kRefillMaxBanks + 1];  // first piece of each bank within a miss; pbase[n] = per miss
    unsigned char vec16[kRefillMaxBanks], vec4[kRefillMaxBanks];
    unsigned char down[kRefillMaxBanks];  // 1: a bank of the down matrix (gate/up banks first)
    int pieces_gu, pieces_dn;             // pieces per miss of the gate/up and of the down banks
    int n_banks;                     // 0: no refill in this call
    int32_t* counts;                 // miss list: [1] misses, [2] status
    const int32_t* miss_ids;
    const int32_t* miss_slots;
    const int32_t* host_slot_of_id;
    int32_t n_gpu_slots;
};

struct FfnParams {
    nvmoe_expert_pool pool;
    nvmoe_expert_pool shared;
    int has_shared;
    const uint16_t* shared_gate;
    const uint16_t* x;
    int64_t x_stride;
    const int32_t* ids;
    int64_t ids_stride;
    const float* w;
    int64_t w_stride;
    int top_k;
    int n_tok;
    uint16_t* y;
    int64_t y_stride;
    unsigned char* ws;
    WsLayout L;
    int32_t* status;
    int grp_tok;           // entries per token group: min(8, n_tok), at least 1
    const uint32_t* aux_table;  // the format's lookup table in device memory (IQ2_XXS grid)
    int kernel;            // enum nvmoe_kernel of the call
    int use_fp4;           // 1: the block-scaled FP4 tensor-core kernel runs this call (NVFP4)
    int spare_sm;          // 1: the FFN grid leaves one SM free (for the next layer's front)
    FfnRefill rf;          // misses this call copies in (rf.n_banks = 0: none)
};

template <typename T>
__device__ __forceinline__ T* wsp(const FfnParams& P, size_t off) {
    return reinterpret_cast<T*>(P.ws + off);
}

#ifdef __CUDACC__
__device__ __forceinline__ float global_of(const nvmoe_matrix_bank& b, int slot) {
    return b.global_scale ? __ldcg(b.global_scale + (int64_t)slot * b.global_stride) : 1.0f;
}
// The same load issued where it stands (not sunk to its first use), for a value needed only at
// the end of a long stretch of work.
// The fields of one matrix bank of the routed pool (sh = 0) or of the shared expert's pool
// (sh = 1), each read at its fixed place in the kernel parameters and then selected as a value
// (selp in inline assembly, so that the choice cannot become a runtime-indexed read of the
// parameter block, which is a memory load on the critical path of a single-lane producer).
struct BankSel {
    const uint8_t* data;
    int64_t slot_stride, row_stride;
    const uint8_t* scale;
    int64_t scale_slot_stride, scale_row_stride;
    const float* global_scale;
    int64_t global_stride;
};
__device__ __forceinline__ int64_t sel64(int c, int64_t a, int64_t b) {  // c ? b : a
    int64_t r;
    asm("{ .reg .pred p; setp.ne.s32 p, %3, 0; selp.b64 %0, %2, %1, p; }"
        : "=l"(r)
        : "l"(a), "l"(b), "r"(c));
    return r;
}
template <typename T>
__device__ __forceinline__ T* selp_ptr(int c, T* a, T* b) {
    return reinterpret_cast<T*>(sel64(c, reinterpret_cast<int64_t>(a), reinterpret_cast<int64_t>(b)));
}
__device__ __forceinline__ BankSel bank_sel(int sh, const nvmoe_matrix_bank& a,
                                            const nvmoe_matrix_bank& b) {
    BankSel r;
    r.data = selp_ptr(sh, static_cast<const uint8_t*>(a.data), static_cast<const uint8_t*>(b.data));
    r.slot_stride = sel64(sh, a.slot_stride, b.slot_stride);
    r.row_stride = sel64(sh, a.row_stride, b.row_stride);
    r.scale = selp_ptr(sh, static_cast<const uint8_t*>(a.scale), static_cast<const uint8_t*>(b.scale));
    r.scale_slot_stride = sel64(sh, a.scale_slot_stride, b.scale_slot_stride);
    r.scale_row_stride = sel64(sh, a.scale_row_stride, b.scale_row_stride);
    r.global_scale = selp_ptr(sh, a.global_scale, b.global_scale);
    r.global_stride = sel64(sh, a.global_stride, b.global_stride);
    return r;
}
// the slot's global scale (1 without a global-scale bank), read through L2
__device__ __forceinline__ float global_of_sel(const BankSel& b, int slot) {
    if (!b.global_scale) return 1.0f;
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];"
                 : "=f"(v)
                 : "l"(b.global_scale + (int64_t)slot * b.global_stride));
    return v;
}
__device__ __forceinline__ float global_of_early(const nvmoe_matrix_bank& b, int slot) {
    if (!b.global_scale) return 1.0f;
    float v;
    asm volatile("ld.global.cg.f32 %0, [%1];"
                 : "=f"(v)
                 : "l"(b.global_scale + (int64_t)slot * b.global_stride));
    return v;
}

// Completes group record d (slot, pool, e0, nt already set): token of each entry, router weight
// of each entry (w_of_entry: the group's entries' weights, or null for the shared expert, whose
// weight is 1 and whose sigmoid gate is applied per token by the down phase), and resets the
// group's completion counter.  No global scale: in a decode layer step the grouping runs
// before the refill that may replace the slot's expert.
__device__ inline void finish_record(const FfnParams& P, int grp, int* d, const int* tok_of_entry,
                                     const float* w_of_entry) {
    const int nt = d[GD_NT];
    float* f = reinterpret_cast<float*>(d);
    for (int k = 0; k < kGroupMaxTok; ++k) {
        d[GD_TOK + k] = k < nt ? tok_of_entry[k] : 0;
        f[GD_W + k] = k < nt ? (w_of_entry ? w_of_entry[k] : 1.0f) : 0.0f;
    }
    d[GD_RT] = 0;
    d[GD_GID] = grp;
    d[14] = d[15] = d[19] = 0;
    f[GD_GGLOB] = f[GD_UGLOB] = f[GD_DGLOB] = 0.f;
    for (int k = 28; k < kDescInts; ++k) d[k] = 0;
    wsp<int>(P, P.L.grp_done)[grp] = 0;
    wsp<int>(P, P.L.gcnt)[2 * grp] = 0;
    wsp<int>(P, P.L.gcnt)[2 * grp + 1] = 0;
}

// Zeroes the grid phase counters of the FP4 kernel (whole block).
__device__ inline void reset_phase_counters(const FfnParams& P) {
    if (threadIdx.x < 4) wsp<int>(P, P.L.phase)[threadIdx.x] = 0;
}

// Power-of-two exponent of an activation row for the FP4 path: |row max| * 2^k in [1024, 2048)
// (k = 0 for a zero, infinite or NaN maximum), kept within +-120 so 2^k and 2^-(k + 6) are
// normal floats.
__host__ __device__ inline int fp4_row_exp(float amax) {
    if (!(amax > 0.f) || !(amax < 3.0e38f)) return 0;
    uint32_t bits;
    memcpy(&bits, &amax, 4);
    const int e = (int)((bits >> 23) & 0xff) - 127;  // floor(log2 amax) for normal values
    const int k = 10 - e;
    return k < -120 ? -120 : (k > 120 ? 120 : k);
}
__host__ __device__ inline float fp4_exp2(int k) {  // 2^k for k in [-126, 127]
    const uint32_t bits = (uint32_t)(k + 127) << 23;
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

// Token rows -> f16 copy (the MMA B operand) and the shared-expert gate sigmoid(x . g), for
// tokens t = t_begin, t_begin + t_step, ... by the whole block.  On the FP4 path: no f16 copy,
// the row's term exponent instead (xk).
__device__ inline void ffn_convert_tokens(const FfnParams& P, int t_begin, int t_step) {
    const int H = P.pool.hidden;
    __shared__ float red[32];
    __shared__ float amx[32];
    for (int t = t_begin; t < P.n_tok; t += t_step) {
        const uint16_t* xr = P.x + (int64_t)t * P.x_stride;
        __half* x16 = wsp<__half>(P, P.L.x16) + (int64_t)t * H;
        float dot = 0.f, amax = 0.f;
        for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
            __align__(16) __half o[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = bf16_bits_to_f32(e[k]);
                o[k] = __float2half_rn(f);
                amax = fmaxf(amax, fabsf(f));
                if (P.shared_gate) dot = fmaf(f, bf16_bits_to_f32(P.shared_gate[i + k]), dot);
            }
            if (!P.use_fp4) *reinterpret_cast<uint4*>(x16 + i) = *reinterpret_cast<const uint4*>(o);
        }
        if (P.use_fp4) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if ((threadIdx.x & 31) == 0) amx[threadIdx.x >> 5] = amax;
            __syncthreads();
            if (threadIdx.x == 0) {
                float m = 0.f;
                for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, amx[w]);
                wsp<int>(P, P.L.xk)[t] = fp4_row_exp(m);
            }
            __syncthreads();
        }
        if (P.shared_gate) {
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = dot;
            __syncthreads();
            if (threadIdx.x == 0) {
                float s = 0.f;
                for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
                wsp<float>(P, P.L.sg)[t] = 1.0f / (1.0f + expf(-s));
            }
            __syncthreads();
        }
    }
}

// Groups the (token, k) entries by slot: active slots ascending, entries of a slot in
// arrival order, token groups of <= 8 consecutive entries with their descriptors, and the
// inverse map ent_of[t*(k+1)+j].  Run by one whole block; smem: n_slots ints.
__device__ inline void ffn_group_block(const FfnParams& P, int* smem_i) {
    const int tid = threadIdx.x, nthr = blockDim.x;
    const int S = P.pool.n_slots;
    int* cnt = smem_i;  // [S]: count, then scatter cursor
    __shared__ int warp_sums[33];
    __shared__ int s_bad;
    const int K = P.top_k;
    const int n = P.n_tok * K;
    __syncthreads();
    if (tid == 0) s_bad = 0;
    for (int s = tid; s < S; s += nthr) cnt[s] = 0;
    reset_phase_counters(P);
    __syncthreads();
    for (int p = tid; p < n; p += nthr) {
        const int t = p / K, j = p - t * K;
        const int s = P.ids[(int64_t)t * P.ids_stride + j];
        if (s >= 0 && s < S)
            atomicAdd(&cnt[s], 1);
        else if (s >= S)
            s_bad = 1;  // (a negative id is an empty entry)
    }
    __syncthreads();
    int* active_slot = wsp<int>(P, P.L.active_slot);
    int* tok_cnt = wsp<int>(P, P.L.tok_cnt);
    int* desc = wsp<int>(P, P.L.grp_desc);
    int n_act = 0, n_ent = 0, n_grp = 0;
    for (int base = 0; base < S; base += nthr) {
        const int s = base + tid;
        const int c = s < S ? cnt[s] : 0;
        const int ng = (c + P.grp_tok - 1) / P.grp_tok;
        int tot_a, tot_e, tot_g;
        const int ra = block_exclusive_scan(c > 0 ? 1 : 0, warp_sums, &tot_a);
        const int re = block_exclusive_scan(c, warp_sums, &tot_e);
        const int rg = block_exclusive_scan(ng, warp_sums, &tot_g);
        if (c > 0) {
            active_slot[n_act + ra] = s;
            tok_cnt[n_act + ra] = c;
            cnt[s] = n_ent + re;  // becomes the scatter cursor
            for (int i = 0; i < ng; ++i) {
                int* d = desc + (int64_t)(n_grp + rg + i) * kDescInts;
                d[GD_SLOT] = s;
                d[GD_POOL] = 0;
                d[GD_E0] = n_ent + re + i * P.grp_tok;
                d[GD_NT] = min(P.grp_tok, c - i * P.grp_tok);
            }
        }
        n_act += tot_a;
        n_ent += tot_e;
        n_grp += tot_g;
    }
    __syncthreads();
    int* ent_tok = wsp<int>(P, P.L.ent_tok);
    float* ent_w = wsp<float>(P, P.L.ent_w);
    int* ent_of = wsp<int>(P, P.L.ent_of);
    for (int p = tid; p < n; p += nthr) {
        const int t = p / K, j = p - t * K;
        const int s = P.ids[(int64_t)t * P.ids_stride + j];
        int e = -1;
        if (s >= 0 && s < S) {
            e = atomicAdd(&cnt[s], 1);
            ent_tok[e] = t;
            ent_w[e] = P.w[(int64_t)t * P.w_stride + j];
        }
        ent_of[t * (K + 1) + j] = e;
    }
    __syncthreads();
    // complete the routed groups' records (the entries of a group are consecutive)
    for (int g = tid; g < n_grp; g += nthr) {
        int* d = desc + (int64_t)g * kDescInts;
        const int e0 = d[GD_E0];
        finish_record(P, g, d, ent_tok + e0, ent_w + e0);
    }
    if (P.has_shared) {
        const int ngs = (P.n_tok + P.grp_tok - 1) / P.grp_tok;
        for (int t = tid; t < P.n_tok; t += nthr) {
            const int e = n_ent + t;
            ent_tok[e] = t;
            ent_w[e] = 1.0f;  // the sigmoid gate is applied by the down phase
            ent_of[t * (K + 1) + K] = e;
        }
        __syncthreads();
        for (int i = tid; i < ngs; i += nthr) {
            int* d = desc + (int64_t)(n_grp + i) * kDescInts;
            const int nt = min(P.grp_tok, P.n_tok - i * P.grp_tok);
            d[GD_SLOT] = 0;
            d[GD_POOL] = 1;
            d[GD_E0] = n_ent + i * P.grp_tok;
            d[GD_NT] = nt;
            finish_record(P, n_grp + i, d, ent_tok + n_ent + i * P.grp_tok, nullptr);
        }
        if (tid == 0) {
            active_slot[n_act] = 0;
            tok_cnt[n_act] = P.n_tok;
        }
        n_act += 1;
        n_ent += P.n_tok;
        n_grp += ngs;
    } else {
        for (int t = tid; t < P.n_tok; t += nthr) ent_of[t * (K + 1) + K] = -1;
    }
    if (tid == 0) {
        int* hdr = wsp<int>(P, P.L.hdr);
        hdr[HDR_N_GROUPS] = n_grp;
        hdr[HDR_N_ACTIVE] = n_act;
        hdr[HDR_N_ENT] = n_ent;
        hdr[HDR_STATUS] = s_bad ? NVMOE_ERR_BAD_SLOT : NVMOE_OK;
        if (P.status) *P.status = s_bad ? NVMOE_ERR_BAD_SLOT : NVMOE_OK;
    }
    __syncthreads();
}
#endif  // __CUDACC__

// Host: fills the kernel-shape part of FfnParams and launches gate_up + down (PDL-chained
// after whatever ran before on `st`, which must have produced the group tables).
int ffn_launch_main(FfnParams& P, cudaStream_t st);
// Host: validates an nvmoe_ffn_args and fills FfnParams (no launch).
int ffn_setup(const nvmoe_ffn_args* args, FfnParams& P);

}  // namespace nvmoe
