// R7 / R9 — routed-expert FFN over the slot pool for decode-sized batches (1..64 tokens).
//
// Reference call: _expert_gemm(cache, hidden, topk_weights, slot_ids, views, n, alphas,
// is_prefill) (nvme-moe-bench/nvme_offload_cache.py:1989-1998, 2165-2174) and ggml mul_mat_id
// over the reduced [.., .., cache_size] expert tensors (scripts/test_mul_mat_id_shrink.cpp:29-69):
//   y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] ),  s = slot_ids[t, j]
// plus the always-on shared expert (nvme_offload_cache.py:2115-2123).
//
// Three kernels chained with programmatic dependent launch:
//   1. prep     : x -> f16, shared-expert gate, grouping of (token, k) entries by slot
//                 (slot histogram, ordered compaction of the active slots, scatter)
//   2. gate_up  : item = (active slot, 16 rows of gate and the matching 16 rows of up); the
//                 8 warps split K; A fragments are dequantised in registers straight from
//                 16-byte streaming loads of the packed slot rows; f16 tensor-core MMA with fp32
//                 accumulation; SwiGLU epilogue writes h (f16) per entry
//   3. down     : item = (active slot, 32 rows of down); y_part[entry] = w * down(h) (fp32);
//                 the last CTA to finish a row block sums the entries of each token in the
//                 fixed order j = 0..k-1, shared, and writes bf16 y (deterministic, no atomics
//                 on the data).
// Only the slots that occur in slot_ids are read; every weight byte is read once per call.
#include "common.cuh"
#include "dequant_frag.cuh"

#include <algorithm>

namespace nvmoe {
namespace {

constexpr int kThreads = 256;  // 8 warps
constexpr int kWarps = kThreads / 32;

// ------------------------------------------------------------------ workspace layout
struct WsLayout {
    size_t hdr, active_slot, active_pool, tok_off, tok_cnt, ent_tok, ent_w, ent_of, x16, sg, h16,
        ypart, row_cnt, total;
    int a_max, n_ent_max, n_rowblk;
};


__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

__host__ __device__ inline WsLayout ws_layout(int n_tok, int top_k, int H, int I, int n_slots) {
    WsLayout L;
    const int n_route = n_tok * top_k;
    L.a_max = (n_route < n_slots ? n_route : n_slots) + 1;
    L.n_ent_max = n_route + n_tok;
    L.n_rowblk = H / 16;  // upper bound on row blocks of the down kernel
    size_t o = 0;
    L.hdr = o;
    o = align_up(o + 64, 256);
    L.active_slot = o;
    o = align_up(o + 4 * (size_t)L.a_max, 256);
    L.active_pool = o;
    o = align_up(o + 4 * (size_t)L.a_max, 256);
    L.tok_off = o;
    o = align_up(o + 4 * (size_t)(L.a_max + 1), 256);
    L.tok_cnt = o;
    o = align_up(o + 4 * (size_t)L.a_max, 256);
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
    L.ypart = o;
    o = align_up(o + 4 * (size_t)L.n_ent_max * H, 256);
    L.row_cnt = o;
    o = align_up(o + 4 * (size_t)L.n_rowblk, 256);
    L.total = o;
    return L;
}

// header words
enum { HDR_N_ACTIVE = 0, HDR_N_ROUTED_ACTIVE = 1, HDR_N_ENT = 2, HDR_STATUS = 3 };

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
    int ks_down;  // K splits of the down kernel (RT = 8 / ks_down row tiles of 16)
};

template <typename T>
__device__ __forceinline__ T* wsp(const FfnParams& P, size_t off) {
    return reinterpret_cast<T*>(P.ws + off);
}

// ------------------------------------------------------------------ 1. prep
__global__ void __launch_bounds__(kThreads) ffn_prep_kernel(FfnParams P) {
    grid_dep_wait();
    grid_dep_launch();
    const int tid = threadIdx.x;
    const int H = P.pool.hidden;
    if ((int)blockIdx.x < P.n_tok) {
        // token row: bf16 -> f16 copy and the shared-expert gate
        const int t = blockIdx.x;
        const uint16_t* xr = P.x + (int64_t)t * P.x_stride;
        __half* x16 = wsp<__half>(P, P.L.x16) + (int64_t)t * H;
        float dot = 0.f;
        for (int i = tid * 8; i < H; i += kThreads * 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
            __align__(16) __half o[8];
#pragma unroll
            for (int k = 0; k < 8; ++k) {
                const float f = bf16_bits_to_f32(e[k]);
                o[k] = __float2half_rn(f);
                if (P.shared_gate) dot = fmaf(f, bf16_bits_to_f32(P.shared_gate[i + k]), dot);
            }
            *reinterpret_cast<uint4*>(x16 + i) = *reinterpret_cast<const uint4*>(o);
        }
        if (P.shared_gate) {
            __shared__ float red[kWarps];
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
            if ((tid & 31) == 0) red[tid >> 5] = dot;
            __syncthreads();
            if (tid == 0) {
                float s = 0.f;
                for (int w = 0; w < kWarps; ++w) s += red[w];
                wsp<float>(P, P.L.sg)[t] = 1.0f / (1.0f + expf(-s));
            }
        }
        return;
    }

    // grouping block
    extern __shared__ __align__(16) int gsm[];
    const int S = P.pool.n_slots;
    int* cnt = gsm;         // [S]
    int* uidx = gsm + S;    // [S]
    __shared__ int warp_sums[33];
    __shared__ int s_bad;
    const int K = P.top_k;
    const int n = P.n_tok * K;
    if (tid == 0) s_bad = 0;
    for (int s = tid; s < S; s += kThreads) cnt[s] = 0;
    for (int i = tid; i < P.L.n_rowblk; i += kThreads) wsp<int>(P, P.L.row_cnt)[i] = 0;
    __syncthreads();
    for (int p = tid; p < n; p += kThreads) {
        const int t = p / K, j = p - t * K;
        const int s = P.ids[(int64_t)t * P.ids_stride + j];
        if (s >= 0 && s < S)
            atomicAdd(&cnt[s], 1);
        else
            s_bad = 1;
    }
    __syncthreads();
    // active slots in ascending order + entry offsets (chunked block scans)
    int* active_slot = wsp<int>(P, P.L.active_slot);
    int* active_pool = wsp<int>(P, P.L.active_pool);
    int* tok_off = wsp<int>(P, P.L.tok_off);
    int* tok_cnt = wsp<int>(P, P.L.tok_cnt);
    int n_act = 0, n_ent = 0;
    for (int base = 0; base < S; base += kThreads) {
        const int s = base + tid;
        const int c = s < S ? cnt[s] : 0;
        int tot_a, tot_e;
        const int ra = block_exclusive_scan(c > 0 ? 1 : 0, warp_sums, &tot_a);
        const int re = block_exclusive_scan(c, warp_sums, &tot_e);
        if (c > 0) {
            const int a = n_act + ra;
            uidx[s] = a;
            active_slot[a] = s;
            active_pool[a] = 0;
            tok_off[a] = n_ent + re;
            tok_cnt[a] = c;
            cnt[s] = n_ent + re;  // becomes the scatter cursor
        }
        n_act += tot_a;
        n_ent += tot_e;
    }
    __syncthreads();
    int* ent_tok = wsp<int>(P, P.L.ent_tok);
    float* ent_w = wsp<float>(P, P.L.ent_w);
    int* ent_of = wsp<int>(P, P.L.ent_of);
    for (int p = tid; p < n; p += kThreads) {
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
    const int n_routed_act = n_act;
    if (P.has_shared) {
        for (int t = tid; t < P.n_tok; t += kThreads) {
            const int e = n_ent + t;
            ent_tok[e] = t;
            ent_w[e] = 1.0f;  // sigmoid gate applied in the down kernel
            ent_of[t * (K + 1) + K] = e;
        }
        if (tid == 0) {
            active_slot[n_act] = 0;
            active_pool[n_act] = 1;
            tok_off[n_act] = n_ent;
            tok_cnt[n_act] = P.n_tok;
        }
        n_act += 1;
        n_ent += P.n_tok;
    } else {
        for (int t = tid; t < P.n_tok; t += kThreads) ent_of[t * (K + 1) + K] = -1;
    }
    if (tid == 0) {
        int* hdr = wsp<int>(P, P.L.hdr);
        hdr[HDR_N_ACTIVE] = n_act;
        hdr[HDR_N_ROUTED_ACTIVE] = n_routed_act;
        hdr[HDR_N_ENT] = n_ent;
        hdr[HDR_STATUS] = s_bad ? NVMOE_ERR_BAD_SLOT : NVMOE_OK;
        if (P.status) *P.status = s_bad ? NVMOE_ERR_BAD_SLOT : NVMOE_OK;
        tok_off[n_act] = n_ent;
    }
}

// ------------------------------------------------------------------ shared helpers
struct ItemInfo {
    int slot, pool, off, cnt;
};
__device__ __forceinline__ ItemInfo item_info(const FfnParams& P, int a) {
    ItemInfo it;
    it.slot = wsp<int>(P, P.L.active_slot)[a];
    it.pool = wsp<int>(P, P.L.active_pool)[a];
    it.off = wsp<int>(P, P.L.tok_off)[a];
    it.cnt = wsp<int>(P, P.L.tok_cnt)[a];
    return it;
}

// ------------------------------------------------------------------ 2. gate_up + SwiGLU
// Warp w owns K range [w*KW, (w+1)*KW) of the 16-row tile; GT groups of 8 tokens per pass.
template <typename Fmt, int GT>
__global__ void __launch_bounds__(kThreads, GT >= 2 ? 1 : 2) ffn_gate_up_kernel(FfnParams P) {
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int KW = H / kWarps;
    const int tiles_per_expert = I / 16;
    const int n_act = wsp<int>(P, P.L.hdr)[HDR_N_ACTIVE];
    const int n_items = n_act * tiles_per_expert;
    const __half* x16 = wsp<__half>(P, P.L.x16);
    const int* ent_tok = wsp<int>(P, P.L.ent_tok);
    __half* h16 = wsp<__half>(P, P.L.h16);

    // cross-warp reduction buffer: [warp][GT][lane][8]
    __shared__ float red[kWarps][GT][32][8];

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int a = item / tiles_per_expert;
        const int rt = item - a * tiles_per_expert;
        const ItemInfo it = item_info(P, a);
        const nvmoe_expert_pool& pool = it.pool ? P.shared : P.pool;
        const uint8_t* gbase = (const uint8_t*)pool.gate.data + it.slot * pool.gate.slot_stride +
                               (int64_t)(rt * 16) * pool.gate.row_stride;
        const uint8_t* ubase = (const uint8_t*)pool.up.data + it.slot * pool.up.slot_stride +
                               (int64_t)(rt * 16) * pool.up.row_stride;
        const uint8_t* gsb = (const uint8_t*)pool.gate.scale + it.slot * pool.gate.scale_slot_stride +
                             (int64_t)(rt * 16) * pool.gate.scale_row_stride;
        const uint8_t* usb = (const uint8_t*)pool.up.scale + it.slot * pool.up.scale_slot_stride +
                             (int64_t)(rt * 16) * pool.up.scale_row_stride;
        const float gglob = pool.gate.global_scale
                                ? pool.gate.global_scale[(int64_t)it.slot * pool.gate.global_stride]
                                : 1.0f;
        const float uglob = pool.up.global_scale
                                ? pool.up.global_scale[(int64_t)it.slot * pool.up.global_stride]
                                : 1.0f;

        for (int t0 = 0; t0 < it.cnt; t0 += 8 * GT) {
            const int ng = min(GT, (it.cnt - t0 + 7) >> 3);
            // token rows of this lane's B fragments (token g of each 8-group)
            const __half* xrow[GT];
#pragma unroll
            for (int gg = 0; gg < GT; ++gg) {
                const int n = t0 + gg * 8 + g;
                xrow[gg] = (n < it.cnt) ? x16 + (int64_t)ent_tok[it.off + n] * H : nullptr;
            }
            float accg[GT][4], accu[GT][4];
#pragma unroll
            for (int gg = 0; gg < GT; ++gg)
#pragma unroll
                for (int v = 0; v < 4; ++v) accg[gg][v] = accu[gg][v] = 0.f;

            for (int k0 = warp * KW; k0 < (warp + 1) * KW; k0 += Fmt::kWarpTileK) {
                typename Fmt::Row ga, gb, ua, ub;  // rows g and g+8 of gate / up
                Fmt::load(ga, gbase + (int64_t)g * pool.gate.row_stride,
                          gsb + (int64_t)g * pool.gate.scale_row_stride, k0, q);
                Fmt::load(gb, gbase + (int64_t)(g + 8) * pool.gate.row_stride,
                          gsb + (int64_t)(g + 8) * pool.gate.scale_row_stride, k0, q);
                Fmt::load(ua, ubase + (int64_t)g * pool.up.row_stride,
                          usb + (int64_t)g * pool.up.scale_row_stride, k0, q);
                Fmt::load(ub, ubase + (int64_t)(g + 8) * pool.up.row_stride,
                          usb + (int64_t)(g + 8) * pool.up.scale_row_stride, k0, q);
#pragma unroll
                for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
                    // B fragments of steps s2, s2+1 (8 consecutive K of this lane)
                    uint4 xb[GT];
#pragma unroll
                    for (int gg = 0; gg < GT; ++gg) {
                        if (gg < ng && xrow[gg])
                            xb[gg] = ldg16(xrow[gg] + k0 + Fmt::kofs(q, s2));
                        else
                            xb[gg] = make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int ss = 0; ss < 2; ++ss) {
                        const int s = s2 + ss;
                        uint32_t ag[4], au[4];
                        Fmt::deq(ga, s, ag[0], ag[2]);
                        Fmt::deq(gb, s, ag[1], ag[3]);
                        Fmt::deq(ua, s, au[0], au[2]);
                        Fmt::deq(ub, s, au[1], au[3]);
#pragma unroll
                        for (int gg = 0; gg < GT; ++gg) {
                            if (gg < ng) {
                                const uint32_t b0 = ss ? xb[gg].z : xb[gg].x;
                                const uint32_t b1 = ss ? xb[gg].w : xb[gg].y;
                                mma_f16_16816(accg[gg], ag, b0, b1);
                                mma_f16_16816(accu[gg], au, b0, b1);
                            }
                        }
                    }
                }
            }
            // cross-warp reduction (the 8 warps hold partial sums over disjoint K ranges)
#pragma unroll
            for (int gg = 0; gg < GT; ++gg) {
#pragma unroll
                for (int v = 0; v < 4; ++v) {
                    red[warp][gg][lane][v] = accg[gg][v];
                    red[warp][gg][lane][4 + v] = accu[gg][v];
                }
            }
            __syncthreads();
            // epilogue: thread -> (group, lane-slot, value) ; 16 rows x 8 tokens x ng groups
            for (int idx = threadIdx.x; idx < ng * 32 * 4; idx += kThreads) {
                const int gg = idx / 128;
                const int l = (idx >> 2) & 31;
                const int v = idx & 3;
                float sg_ = 0.f, su_ = 0.f;
#pragma unroll
                for (int w = 0; w < kWarps; ++w) {
                    sg_ += red[w][gg][l][v];
                    su_ += red[w][gg][l][4 + v];
                }
                // C fragment position: row = l/4 (+8 for v>=2), token = 2*(l%4) + (v&1)
                const int row = (l >> 2) + ((v >> 1) << 3);
                const int n = t0 + gg * 8 + 2 * (l & 3) + (v & 1);
                if (n < it.cnt) {
                    const float gv = sg_ * gglob;
                    const float uv = su_ * uglob;
                    const float hv = silu(gv) * uv;
                    h16[(int64_t)(it.off + n) * I + rt * 16 + row] = __float2half_rn(hv);
                }
            }
            __syncthreads();
        }
    }
}

// ------------------------------------------------------------------ 3. down + combine
template <typename Fmt, int GT>
__global__ void __launch_bounds__(kThreads, GT >= 4 ? 1 : 2) ffn_down_kernel(FfnParams P) {
    grid_dep_wait();
    grid_dep_launch();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, q = lane & 3;
    const int H = P.pool.hidden, I = P.pool.inter;
    const int KS = P.ks_down, RT = kWarps / KS;
    const int rows_per_item = 16 * RT;
    const int rt = warp % RT, ks = warp / RT;
    const int KW = I / KS;
    const int blocks_per_expert = H / rows_per_item;
    const int* hdr = wsp<int>(P, P.L.hdr);
    const int n_act = hdr[HDR_N_ACTIVE];
    const int n_items = n_act * blocks_per_expert;
    const __half* h16 = wsp<__half>(P, P.L.h16);
    const float* ent_w = wsp<float>(P, P.L.ent_w);
    const int* ent_tok = wsp<int>(P, P.L.ent_tok);
    const int* ent_of = wsp<int>(P, P.L.ent_of);
    float* ypart = wsp<float>(P, P.L.ypart);
    int* row_cnt = wsp<int>(P, P.L.row_cnt);
    const float* sg = P.shared_gate ? wsp<float>(P, P.L.sg) : nullptr;

    __shared__ float red[kWarps][GT][32][4];
    __shared__ int s_last;

    if (n_act == 0) {  // every slot id was invalid and there is no shared expert: y = 0
        for (int64_t i = blockIdx.x * (int64_t)kThreads + threadIdx.x; i < (int64_t)P.n_tok * H;
             i += (int64_t)gridDim.x * kThreads) {
            const int64_t t = i / H;
            P.y[t * P.y_stride + (i - t * H)] = 0;
        }
        return;
    }

    for (int item = blockIdx.x; item < n_items; item += gridDim.x) {
        const int a = item / blocks_per_expert;
        const int rb = item - a * blocks_per_expert;
        const ItemInfo it = item_info(P, a);
        const nvmoe_expert_pool& pool = it.pool ? P.shared : P.pool;
        const int row0 = rb * rows_per_item + rt * 16;
        const uint8_t* dbase = (const uint8_t*)pool.down.data + it.slot * pool.down.slot_stride +
                               (int64_t)row0 * pool.down.row_stride;
        const uint8_t* dsb = (const uint8_t*)pool.down.scale + it.slot * pool.down.scale_slot_stride +
                             (int64_t)row0 * pool.down.scale_row_stride;
        const float dglob = pool.down.global_scale
                                ? pool.down.global_scale[(int64_t)it.slot * pool.down.global_stride]
                                : 1.0f;

        for (int t0 = 0; t0 < it.cnt; t0 += 8 * GT) {
            const int ng = min(GT, (it.cnt - t0 + 7) >> 3);
            const __half* hrow[GT];
#pragma unroll
            for (int gg = 0; gg < GT; ++gg) {
                const int n = t0 + gg * 8 + g;
                hrow[gg] = (n < it.cnt) ? h16 + (int64_t)(it.off + n) * I : nullptr;
            }
            float acc[GT][4];
#pragma unroll
            for (int gg = 0; gg < GT; ++gg)
#pragma unroll
                for (int v = 0; v < 4; ++v) acc[gg][v] = 0.f;

            for (int k0 = ks * KW; k0 < (ks + 1) * KW; k0 += Fmt::kWarpTileK) {
                typename Fmt::Row ra, rbw;
                Fmt::load(ra, dbase + (int64_t)g * pool.down.row_stride,
                          dsb + (int64_t)g * pool.down.scale_row_stride, k0, q);
                Fmt::load(rbw, dbase + (int64_t)(g + 8) * pool.down.row_stride,
                          dsb + (int64_t)(g + 8) * pool.down.scale_row_stride, k0, q);
#pragma unroll
                for (int s2 = 0; s2 < Fmt::kSteps; s2 += 2) {
                    uint4 hb[GT];
#pragma unroll
                    for (int gg = 0; gg < GT; ++gg) {
                        if (gg < ng && hrow[gg])
                            hb[gg] = ldg16(hrow[gg] + k0 + Fmt::kofs(q, s2));
                        else
                            hb[gg] = make_uint4(0, 0, 0, 0);
                    }
#pragma unroll
                    for (int ss = 0; ss < 2; ++ss) {
                        const int s = s2 + ss;
                        uint32_t af[4];
                        Fmt::deq(ra, s, af[0], af[2]);
                        Fmt::deq(rbw, s, af[1], af[3]);
#pragma unroll
                        for (int gg = 0; gg < GT; ++gg)
                            if (gg < ng)
                                mma_f16_16816(acc[gg], af, ss ? hb[gg].z : hb[gg].x,
                                              ss ? hb[gg].w : hb[gg].y);
                    }
                }
            }
#pragma unroll
            for (int gg = 0; gg < GT; ++gg)
#pragma unroll
                for (int v = 0; v < 4; ++v) red[warp][gg][lane][v] = acc[gg][v];
            __syncthreads();
            // sum the K splits; scale; write y_part rows of this item
            for (int idx = threadIdx.x; idx < RT * ng * 128; idx += kThreads) {
                const int rr = idx / (ng * 128);
                const int rem = idx - rr * ng * 128;
                const int gg = rem / 128;
                const int l = (rem >> 2) & 31;
                const int v = rem & 3;
                float s = 0.f;
                for (int kk = 0; kk < KS; ++kk) s += red[kk * RT + rr][gg][l][v];
                const int row = rb * rows_per_item + rr * 16 + (l >> 2) + ((v >> 1) << 3);
                const int n = t0 + gg * 8 + 2 * (l & 3) + (v & 1);
                if (n < it.cnt) {
                    const int e = it.off + n;
                    float wgt = ent_w[e];
                    if (it.pool && sg) wgt *= sg[ent_tok[e]];
                    ypart[(int64_t)e * H + row] = s * dglob * wgt;
                }
            }
            __syncthreads();
        }

        // completion count of this row block; the last item reduces it
        __threadfence();  // every thread's y_part stores are device-visible before the count
        __syncthreads();
        if (threadIdx.x == 0) {
            const int old = atomicAdd(&row_cnt[rb], 1);
            s_last = (old == n_act - 1);
        }
        __syncthreads();
        if (s_last) {
            __threadfence();
            const int K1 = P.top_k + 1;
            for (int idx = threadIdx.x; idx < P.n_tok * rows_per_item; idx += kThreads) {
                const int t = idx / rows_per_item;
                const int row = rb * rows_per_item + (idx - t * rows_per_item);
                float s = 0.f;
                for (int j = 0; j < K1; ++j) {
                    const int e = ent_of[t * K1 + j];
                    if (e >= 0) s += __ldcg(ypart + (int64_t)e * H + row);
                }
                P.y[(int64_t)t * P.y_stride + row] = f32_to_bf16_bits(s);
            }
            if (threadIdx.x == 0) row_cnt[rb] = 0;
        }
        __syncthreads();
    }
}

// ------------------------------------------------------------------ host dispatch
bool pool_ok(const nvmoe_expert_pool& p) {
    return p.gate.data && p.up.data && p.down.data && p.hidden > 0 && p.inter > 0 &&
           p.n_slots > 0;
}

// The kernels read packed rows with 16-byte loads and NVFP4 scale pairs with 2-byte loads;
// reject any bank whose base or strides would break that alignment.
bool bank_aligned(const nvmoe_matrix_bank& b, bool nvfp4) {
    const uintptr_t d = reinterpret_cast<uintptr_t>(b.data);
    if ((d & 15) || (b.slot_stride & 15) || (b.row_stride & 15)) return false;
    if (nvfp4) {
        const uintptr_t s = reinterpret_cast<uintptr_t>(b.scale);
        if (!b.scale || (s & 1) || (b.scale_slot_stride & 1) || (b.scale_row_stride & 1))
            return false;
    }
    return true;
}

bool pool_aligned(const nvmoe_expert_pool& p) {
    const bool nv = p.quant == NVMOE_Q_NVFP4;
    return bank_aligned(p.gate, nv) && bank_aligned(p.up, nv) && bank_aligned(p.down, nv);
}

template <typename Fmt>
int launch_fmt(FfnParams& P, cudaStream_t st, int grid_gu, int grid_dn) {
    const int gt = P.n_tok <= 8 ? 1 : (P.n_tok <= 16 ? 2 : 4);
    cudaError_t e = cudaSuccess;
#define NVMOE_LAUNCH_GT(GTV)                                                                   \
    do {                                                                                       \
        e = launch_pdl(ffn_gate_up_kernel<Fmt, GTV>, dim3(grid_gu), dim3(kThreads), 0, st,     \
                       true, P);                                                               \
        if (e == cudaSuccess)                                                                  \
            e = launch_pdl(ffn_down_kernel<Fmt, GTV>, dim3(grid_dn), dim3(kThreads), 0, st,    \
                           true, P);                                                           \
    } while (0)
    if (gt == 1)
        NVMOE_LAUNCH_GT(1);
    else if (gt == 2)
        NVMOE_LAUNCH_GT(2);
    else
        NVMOE_LAUNCH_GT(4);
#undef NVMOE_LAUNCH_GT
    return cuda_status("ffn launch", e);
}

}  // namespace
}  // namespace nvmoe

extern "C" size_t nvmoe_moe_ffn_workspace_size(int n_tok, int top_k, int hidden, int inter,
                                               int n_slots) {
    if (n_tok <= 0 || top_k <= 0 || hidden <= 0 || inter <= 0 || n_slots <= 0) return 0;
    return nvmoe::ws_layout(n_tok, top_k, hidden, inter, n_slots).total;
}

extern "C" int nvmoe_moe_ffn(const nvmoe_ffn_args* args, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!args || !args->pool || !args->x || !args->slot_ids || !args->weights || !args->y)
        return NVMOE_ERR_INVALID_ARG;
    const nvmoe_expert_pool& pool = *args->pool;
    if (!pool_ok(pool)) return NVMOE_ERR_INVALID_ARG;
    if (args->n_tok < 0 || args->top_k <= 0) return NVMOE_ERR_INVALID_ARG;
    if (args->n_tok == 0) return NVMOE_OK;
    const int H = pool.hidden, I = pool.inter;
    if (args->shared) {
        const nvmoe_expert_pool& sp = *args->shared;
        if (!pool_ok(sp) || sp.quant != pool.quant || sp.hidden != H || sp.inter != I)
            return NVMOE_ERR_INVALID_ARG;
    }
    if (pool.quant != NVMOE_Q_NVFP4) return NVMOE_ERR_UNSUPPORTED;
    // shape rules of the warp tiling: gate_up K = H split over 8 warps, down K = I split over 4
    if (H % (kWarps * FmtNvfp4::kWarpTileK) != 0 || I % 16 != 0) return NVMOE_ERR_UNSUPPORTED;
    int ks_down = 0;
    for (int ks : {4, 2, 8, 1})
        if (I % (ks * FmtNvfp4::kWarpTileK) == 0 && H % (16 * (kWarps / ks)) == 0) {
            ks_down = ks;
            break;
        }
    if (!ks_down) return NVMOE_ERR_UNSUPPORTED;
    if (!pool.gate.scale || !pool.up.scale || !pool.down.scale) return NVMOE_ERR_INVALID_ARG;
    if (!pool_aligned(pool) || (args->shared && !pool_aligned(*args->shared)))
        return NVMOE_ERR_INVALID_ARG;
    // rows must hold exactly K values: H/2 code bytes, H/16 scales (gate/up), I/2, I/16 (down)
    if (pool.gate.row_stride < H / 2 || pool.down.row_stride < I / 2 ||
        pool.gate.scale_row_stride < H / 16 || pool.down.scale_row_stride < I / 16)
        return NVMOE_ERR_INVALID_ARG;
    if (args->x_row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(args->x) & 15))
        return NVMOE_ERR_INVALID_ARG;

    const WsLayout L = ws_layout(args->n_tok, args->top_k, H, I, pool.n_slots);
    if (!args->workspace || args->workspace_bytes < L.total) return NVMOE_ERR_WORKSPACE;

    FfnParams P;
    P.pool = pool;
    P.has_shared = args->shared ? 1 : 0;
    if (args->shared) P.shared = *args->shared; else P.shared = pool;
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
    P.ks_down = ks_down;

    cudaStream_t st = (cudaStream_t)stream;
    const size_t prep_smem = (size_t)pool.n_slots * 8;
    if (prep_smem > 48 * 1024) {
        if (prep_smem > 200 * 1024) return NVMOE_ERR_UNSUPPORTED;
        NVMOE_CUDA_TRY(cudaFuncSetAttribute(ffn_prep_kernel,
                                            cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)prep_smem));
    }
    cudaError_t e = launch_pdl(ffn_prep_kernel, dim3(args->n_tok + 1), dim3(kThreads), prep_smem,
                               st, true, P);
    if (e != cudaSuccess) return cuda_status("ffn_prep launch", e);
    const int items_gu = L.a_max * (I / 16);
    const int items_dn = L.a_max * (H / (16 * (kWarps / ks_down)));
    const int cap = kNumSMs * 4;
    return launch_fmt<FmtNvfp4>(P, st, std::min(items_gu, cap), std::min(items_dn, cap));
}
