// (f)3 tail pruning of one token's routed experts, eval_cb's "two-tier cost-aware expert
// pruning" (scripts/moe_cache_probe.cpp:523-625), as a function the device kernel (prune.cu)
// runs per token row and host code can compile unchanged.
//
// Per row, with total = the sum of the row's router weights (nothing happens unless > 1e-6) and
// rel = weight / total: experts resident in the slot pool are never pruned; walking the picks
// from the last to the first while more than min_keep remain, an expert only in the host tier
// is pruned if host_thresh > 0, rel < host_thresh and the kept mass stays >= min_mass; an
// expert in neither tier is pruned if (rel < nvme_thresh or the row's resident mass (slot pool
// or host tier) is already >= min_mass) and the kept mass stays >= min_mass.  A pruned pick gets
// weight 0 and the id of the row's first slot-resident expert (else resident_real, the expert of
// the pool's first occupied slot), so it costs no copy; if anything was pruned the weights are
// scaled back to the original total.  Every operation is a single IEEE fp32 operation in the
// reference's order (no fused multiply-add), so results are bit-identical to the host code.
#pragma once

#include <stdint.h>

#ifdef __CUDACC__
#define NVMOE_HD __host__ __device__ __forceinline__
#else
#define NVMOE_HD inline
#endif

namespace nvmoe {

struct PruneCfg {
    float nvme_thresh, host_thresh, min_mass;
    int min_keep;
};

NVMOE_HD float pr_add(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fadd_rn(a, b);
#else
    return a + b;
#endif
}
NVMOE_HD float pr_sub(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fsub_rn(a, b);
#else
    return a - b;
#endif
}
NVMOE_HD float pr_mul(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fmul_rn(a, b);
#else
    return a * b;
#endif
}
NVMOE_HD float pr_div(float a, float b) {
#ifdef __CUDA_ARCH__
    return __fdiv_rn(a, b);
#else
    return a / b;
#endif
}

// ids / w: the row's k picks (ids already checked to lie in the tables); host_slot_of_real may
// be null (no host tier).  pruned[0] / pruned[1] count the picks pruned from the backing store
// tier / the host tier.
NVMOE_HD void prune_row(int32_t* ids, float* w, int k, const int32_t* slot_of_real,
                        const int32_t* host_slot_of_real, int32_t resident_real,
                        const PruneCfg& c, int* pruned) {
    float total = 0.0f;
    for (int i = 0; i < k; ++i) total = pr_add(total, w[i]);
    if (!(total > 1e-6f)) return;
    int32_t row_gpu_resident = -1;
    float in_mem_mass = 0.0f;
    for (int i = 0; i < k; ++i) {
        const int32_t rid = ids[i];
        const bool in_gpu = slot_of_real[rid] != -1;
        const bool in_host = host_slot_of_real && host_slot_of_real[rid] != -1;
        if (in_gpu && row_gpu_resident == -1) row_gpu_resident = rid;
        if (in_gpu || in_host) in_mem_mass = pr_add(in_mem_mass, pr_div(w[i], total));
    }
    const int32_t alias_target = row_gpu_resident != -1 ? row_gpu_resident : resident_real;
    float remaining_mass = 1.0f;
    int kept = k;
    bool modified = false;
    for (int j = k - 1; j >= 0; --j) {
        if (kept <= c.min_keep) break;
        const int32_t rid = ids[j];
        const bool in_gpu = slot_of_real[rid] != -1;
        const bool in_host = host_slot_of_real && host_slot_of_real[rid] != -1;
        if (in_gpu) continue;
        const float rel = pr_div(w[j], total);
        if (in_host) {
            if (c.host_thresh > 0.0f && rel < c.host_thresh &&
                pr_sub(remaining_mass, rel) >= c.min_mass) {
                w[j] = 0.0f;
                ids[j] = alias_target;
                remaining_mass = pr_sub(remaining_mass, rel);
                --kept;
                modified = true;
                ++pruned[1];
            }
            continue;
        }
        const bool should = (rel < c.nvme_thresh) || (in_mem_mass >= c.min_mass);
        if (should && pr_sub(remaining_mass, rel) >= c.min_mass) {
            w[j] = 0.0f;
            ids[j] = alias_target;
            remaining_mass = pr_sub(remaining_mass, rel);
            --kept;
            modified = true;
            ++pruned[0];
        }
    }
    if (modified) {
        float new_total = 0.0f;
        for (int i = 0; i < k; ++i) new_total = pr_add(new_total, w[i]);
        if (new_total > 1e-6f) {
            const float f = pr_div(total, new_total);
            for (int i = 0; i < k; ++i) w[i] = pr_mul(w[i], f);
        }
    }
}

}  // namespace nvmoe
