// R1 router top-k, warp-level device function shared by the router kernel and the fused decode
// front kernel (see router.cu for the reference behaviour).
#pragma once

#include "common.cuh"

namespace nvmoe {

constexpr int kMaxExperts = 1024;
constexpr int kPerLane = kMaxExperts / 32;
constexpr int kMaxTopK = 32;

__device__ __forceinline__ bool key_better(float ka, int ia, float kb, int ib) {
    return ka > kb || (ka == kb && ia < ib);
}

// Top-k of one token row by one warp; writes ids / weights [top_k] (called by all 32 lanes).
__device__ __forceinline__ void router_topk_warp(const float* __restrict__ lr, int n_expert,
                                                 int top_k, int mode,
                                                 const float* __restrict__ bias, int norm_topk,
                                                 float scaling, int32_t* __restrict__ ids_row,
                                                 float* __restrict__ w_row) {
    const int lane = threadIdx.x & 31;

    float key[kPerLane];
    float val[kPerLane];  // softmax: logit; sigmoid: score
#pragma unroll
    for (int i = 0; i < kPerLane; ++i) {
        const int e = i * 32 + lane;
        float k = -INFINITY, v = -INFINITY;
        if (e < n_expert) {
            float l = lr[e];
            if (mode == NVMOE_ROUTER_SOFTMAX) {
                v = l;
                k = (l != l) ? -INFINITY : l;  // NaN logits never win
            } else {
                float s = 1.0f / (1.0f + expf(-l));
                v = s;
                float c = s + (bias ? bias[e] : 0.0f);
                k = (c != c) ? -INFINITY : c;
            }
        }
        key[i] = k;
        val[i] = v;
    }

    // Lane j keeps the j-th pick (top_k <= 32), so no per-thread arrays spill to local memory.
    float my_val = 0.f, first_val = 0.f;
    int my_id = -1;
    uint32_t taken = 0;  // bit i: expert i*32+lane already chosen
    for (int j = 0; j < top_k; ++j) {
        float bk = -INFINITY;
        int bi = 0x7fffffff;
        float bv = 0.f;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int e = i * 32 + lane;
            if (e < n_expert && !((taken >> i) & 1u) && key_better(key[i], e, bk, bi)) {
                bk = key[i];
                bi = e;
                bv = val[i];
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            float ok = __shfl_xor_sync(0xffffffffu, bk, o);
            int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            if (key_better(ok, oi, bk, bi)) {
                bk = ok;
                bi = oi;
                bv = ov;
            }
        }
        if (lane == j) my_id = bi, my_val = bv;
        if (j == 0) first_val = bv;
        if ((bi & 31) == lane) taken |= 1u << (bi >> 5);
    }

    // Full-softmax denominator (only when the top-k weights are not renormalised).
    float full_denom = 0.f;
    if (mode == NVMOE_ROUTER_SOFTMAX && !norm_topk) {
        const float m = first_val;
#pragma unroll
        for (int i = 0; i < kPerLane; ++i) {
            const int e = i * 32 + lane;
            if (e < n_expert && val[i] == val[i]) full_denom += expf(val[i] - m);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) full_denom += __shfl_xor_sync(0xffffffffu, full_denom, o);
    }

    const bool mine = lane < top_k;
    float w;
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        // probabilities relative to the row maximum (= the first pick)
        w = mine ? expf(my_val - first_val) : 0.f;
    } else {
        w = mine ? my_val : 0.f;
    }
    // sum of the picks in pick order (lane 0 first), identical on every lane
    float sum = 0.f;
    for (int j = 0; j < top_k; ++j) sum += __shfl_sync(0xffffffffu, w, j);
    if (mode == NVMOE_ROUTER_SOFTMAX) {
        const float denom = norm_topk ? sum : full_denom;
        w = w / denom * scaling;
    } else {
        w = (norm_topk ? w / (sum + 1e-20f) : w) * scaling;
    }
    if (mine) {
        ids_row[lane] = my_id;
        w_row[lane] = w;
    }
}


}  // namespace nvmoe
