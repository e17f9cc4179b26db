// Expert parallelism: pack a rank's tokens for the owners of their experts, and sum the owners'
// outputs back (nvmoe_ep_dispatch / nvmoe_ep_combine).
//
// The reference runs on one GPU and has no counterpart; the step these kernels bracket is its
// expert GEMM (_expert_gemm, nvme-moe-bench/nvme_offload_cache.py:2165-2174) split by expert
// range across ranks.  Segments have a fixed size (n_tok rows per destination: a token goes to a
// rank at most once), so the exchange between the two kernels is an all-to-all of equal parts
// and nothing waits for a count on the host.
//
// dispatch: kernel A, one CTA per destination rank d: a block scan over the tokens of "token t
//   goes to d" gives each token its row in segment d; the CTA writes slot_of[., d] and the rows'
//   expert ids and weights (every id -1 in rows past the segment's count).  Kernel B, one CTA
//   per (token, destination) with a row: copies the token (16-byte vectors) and, for the shared
//   expert on this rank, computes sigmoid(x . shared_gate) as that entry's weight.
// combine: one thread per 8 columns of a token: the world segments' rows in rank order, fp32,
//   bf16 out (a fixed order: the result does not depend on scheduling).
#include "common.cuh"

#include <algorithm>

namespace nvmoe {
namespace {

constexpr int kScanThreads = 1024;

__host__ __device__ inline size_t ep_row_bytes(int H, int k) {
    const size_t b = (size_t)H * 2 + (size_t)(k + 1) * 8;
    return (b + 15) & ~(size_t)15;
}

struct EpDispatch {
    nvmoe_ep_dispatch_args a;
    int64_t row;  // bytes per send row
    int per;      // experts per rank
};

__device__ __forceinline__ int32_t* row_ids(const EpDispatch& D, int d, int slot) {
    unsigned char* r = D.a.send + ((int64_t)d * D.a.n_tok + slot) * D.row;
    return reinterpret_cast<int32_t*>(r + (int64_t)D.a.hidden * 2);
}

__global__ void __launch_bounds__(kScanThreads) ep_dispatch_meta(EpDispatch D) {
    __shared__ int warp_sums[33];
    const nvmoe_ep_dispatch_args& a = D.a;
    const int d = blockIdx.x, K = a.top_k, K1 = K + 1;
    const bool shared_here = a.with_shared && d == a.rank;
    grid_dep_wait();  // the routed ids come from the kernels before this one
    int run = 0;
    for (int base = 0; base < a.n_tok; base += blockDim.x) {
        const int t = base + threadIdx.x;
        bool go = false;
        if (t < a.n_tok) {
            go = shared_here;
            for (int j = 0; j < K; ++j) {
                const int e = a.ids[(int64_t)t * K + j];
                if (e < 0 || e >= a.n_expert) {
                    if (a.status) *a.status = NVMOE_ERR_BAD_EXPERT_ID;
                    continue;
                }
                go |= e / D.per == d;
            }
        }
        int total;
        const int ex = block_exclusive_scan(go ? 1 : 0, warp_sums, &total);
        if (t < a.n_tok) {
            const int slot = go ? run + ex : -1;
            a.slot_of[(int64_t)t * a.world + d] = slot;
            if (go) {
                int32_t* ids = row_ids(D, d, slot);
                float* w = reinterpret_cast<float*>(ids + K1);
                for (int j = 0; j < K; ++j) {
                    const int e = a.ids[(int64_t)t * K + j];
                    const bool mine = e >= 0 && e < a.n_expert && e / D.per == d;
                    ids[j] = mine ? e - d * D.per : -1;
                    w[j] = mine ? a.weights[(int64_t)t * K + j] : 0.f;
                }
                ids[K] = shared_here ? D.per : -1;
                w[K] = shared_here ? 1.0f : 0.f;  // the gate, if any, is written by kernel B
            }
        }
        run += total;
    }
    // rows past the segment's count: no entry
    for (int slot = run + threadIdx.x; slot < a.n_tok; slot += blockDim.x) {
        int32_t* ids = row_ids(D, d, slot);
        for (int j = 0; j < K1; ++j) ids[j] = -1;
    }
}

__global__ void __launch_bounds__(256) ep_dispatch_rows(EpDispatch D) {
    const nvmoe_ep_dispatch_args& a = D.a;
    const int t = blockIdx.x, d = blockIdx.y, H = a.hidden;
    grid_dep_wait();
    const int slot = a.slot_of[(int64_t)t * a.world + d];
    if (slot < 0) return;
    const uint16_t* xr = a.x + (int64_t)t * a.x_row_stride;
    uint16_t* dst = reinterpret_cast<uint16_t*>(a.send + ((int64_t)d * a.n_tok + slot) * D.row);
    const bool gate = a.with_shared && d == a.rank && a.shared_gate;
    float dot = 0.f;
    for (int i = threadIdx.x * 8; i < H; i += blockDim.x * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
        *reinterpret_cast<uint4*>(dst + i) = v;
        if (gate) {
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
            const uint4 g4 = *reinterpret_cast<const uint4*>(a.shared_gate + i);
            const uint16_t* g = reinterpret_cast<const uint16_t*>(&g4);
#pragma unroll
            for (int k = 0; k < 8; ++k) dot = fmaf(bf16_bits_to_f32(e[k]), bf16_bits_to_f32(g[k]), dot);
        }
    }
    if (!gate) return;
    __shared__ float part[8];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, o);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = dot;
    __syncthreads();
    if (threadIdx.x == 0) {
        float s = 0.f;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += part[w];
        int32_t* ids = row_ids(D, d, slot);
        reinterpret_cast<float*>(ids + a.top_k + 1)[a.top_k] = 1.0f / (1.0f + expf(-s));
    }
}

__global__ void __launch_bounds__(256) ep_combine_kernel(nvmoe_ep_combine_args a) {
    grid_dep_wait();  // the returned rows come from the exchange before this kernel
    const int H = a.hidden;
    const int64_t n8 = (int64_t)a.n_tok * (H / 8);
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / (H / 8)), c = (int)(i % (H / 8)) * 8;
        float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int d = 0; d < a.world; ++d) {
            const int slot = a.slot_of[(int64_t)t * a.world + d];
            if (slot < 0) continue;
            const uint4 v =
                *reinterpret_cast<const uint4*>(a.back + ((int64_t)d * a.n_tok + slot) * H + c);
            const uint16_t* e = reinterpret_cast<const uint16_t*>(&v);
#pragma unroll
            for (int k = 0; k < 8; ++k) s[k] += bf16_bits_to_f32(e[k]);
        }
        __align__(16) uint16_t o[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) o[k] = f32_to_bf16_bits(s[k]);
        *reinterpret_cast<uint4*>(a.y + (int64_t)t * a.y_row_stride + c) =
            *reinterpret_cast<const uint4*>(o);
    }
}

}  // namespace
}  // namespace nvmoe

extern "C" size_t nvmoe_ep_row_bytes(int hidden, int top_k) {
    if (hidden <= 0 || top_k <= 0) return 0;
    return nvmoe::ep_row_bytes(hidden, top_k);
}

extern "C" int nvmoe_ep_dispatch(const nvmoe_ep_dispatch_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->x || !a->ids || !a->weights || !a->send || !a->slot_of) return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok < 0 || a->top_k <= 0 || a->hidden <= 0 || a->hidden % 8 != 0 ||
        a->world <= 0 || a->rank < 0 || a->rank >= a->world || a->n_expert < a->world ||
        a->n_expert % a->world != 0 || a->x_row_stride % 8 != 0 ||
        (reinterpret_cast<uintptr_t>(a->x) & 15) || (reinterpret_cast<uintptr_t>(a->send) & 15) ||
        (a->shared_gate && (reinterpret_cast<uintptr_t>(a->shared_gate) & 15)))
        return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok == 0) return NVMOE_OK;
    if (a->n_tok > 65535 || a->world > 65535) return NVMOE_ERR_UNSUPPORTED;
    EpDispatch D;
    D.a = *a;
    D.row = (int64_t)ep_row_bytes(a->hidden, a->top_k);
    D.per = a->n_expert / a->world;
    cudaStream_t st = (cudaStream_t)stream;
    const int threads = std::min(kScanThreads, std::max(32, (a->n_tok + 31) / 32 * 32));
    cudaError_t e = launch_pdl(ep_dispatch_meta, dim3(a->world), dim3(threads), 0, st, true, D);
    if (e != cudaSuccess) return cuda_status("ep_dispatch_meta launch", e);
    e = launch_pdl(ep_dispatch_rows, dim3(a->n_tok, a->world), dim3(256), 0, st, true, D);
    return cuda_status("ep_dispatch_rows launch", e);
}

extern "C" int nvmoe_ep_combine(const nvmoe_ep_combine_args* a, nvmoe_stream_t stream) {
    using namespace nvmoe;
    if (!a || !a->back || !a->slot_of || !a->y) return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok < 0 || a->hidden <= 0 || a->hidden % 8 != 0 || a->world <= 0 ||
        a->y_row_stride % 8 != 0 || (reinterpret_cast<uintptr_t>(a->y) & 15) ||
        (reinterpret_cast<uintptr_t>(a->back) & 15))
        return NVMOE_ERR_INVALID_ARG;
    if (a->n_tok == 0) return NVMOE_OK;
    const int64_t n8 = (int64_t)a->n_tok * (a->hidden / 8);
    const int grid = (int)std::min<int64_t>(8 * kNumSMs, (n8 + 255) / 256);
    const cudaError_t e = launch_pdl(ep_combine_kernel, dim3(grid), dim3(256), 0,
                                     (cudaStream_t)stream, true, *a);
    return cuda_status("ep_combine launch", e);
}
