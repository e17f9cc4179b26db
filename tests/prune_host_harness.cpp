// Host build of the device pruning row function (nvmoe_b200/csrc/prune_device.cuh) for the CPU
// test: the same per-row wrapper as prune.cu's kernel (alias of last resort, id range check,
// decode counters), compiled by g++ without fused multiply-add.
#include <cstdint>

#include "../nvmoe_b200/csrc/prune_device.cuh"

extern "C" void prune_rows_host(int32_t* ids, float* w, int n_tok, int k, const int32_t* sor,
                                const int32_t* hsor, const int32_t* ris, int cache_size,
                                int n_expert, float nvme, float host, float min_mass,
                                int min_keep, int is_decode, int* pruned) {
    if (!(nvme > 0.0f) || (long)n_tok * k > 4096) return;
    int32_t resident_real = -1;
    for (int s = 0; s < cache_size && resident_real == -1; ++s) resident_real = ris[s];
    if (resident_real == -1) return;
    nvmoe::PruneCfg c{nvme, host, min_mass, min_keep};
    for (int t = 0; t < n_tok; ++t) {
        int32_t* ri = ids + (long)t * k;
        bool ok = true;
        for (int i = 0; i < k; ++i) ok = ok && ri[i] >= 0 && ri[i] < n_expert;
        if (!ok) continue;
        int p[2] = {0, 0};
        nvmoe::prune_row(ri, w + (long)t * k, k, sor, hsor, resident_real, c, p);
        if (is_decode) pruned[0] += p[0], pruned[1] += p[1];
    }
}
