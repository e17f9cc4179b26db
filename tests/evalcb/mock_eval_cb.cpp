// Mock llama.cpp scheduler driving libnvmoe_b200 through its C ABI (include/nvmoe_b200.h) the
// way the reference's eval callback is driven by ggml_backend_sched
// (scripts/moe_cache_probe.cpp:439-997) and exercised by scripts/test_sched_chain_shrink.cpp:
//   - the callback is asked per node and claims GET_ROWS nodes named "ffn_moe_weights-N"
//     (moe_cache_probe.cpp:474-488);
//   - it reads the node's src[1], the selected-experts view [n_expert_used, n_tokens] whose rows
//     are nb[1] = n_as_full * 4 bytes apart (a column slice of the argsort output,
//     test_sched_chain_shrink.cpp:75-105,211-215), rewrites it in place to slot ids
//     (nvmoe_remap with the byte row stride), reads the miss list back to the host and copies
//     the missed experts from the pinned host tier on a high-priority side stream joined to the
//     compute stream by an event (nvmoe_refill_async; moe_cache_probe.cpp:755-784,988-993);
//   - the "mul_mat_id" node then runs the expert FFN on the slot-sized pool (nvmoe_moe_ffn),
//     reading the rewritten ids through the same strided view;
//   - two MoE layers are chained: layer l + 1's tokens are RMSNorm(x_l + y_l) of layer l's input
//     and output (nvmoe_router_gate with no gate matrix), as a decoder stack feeds them.
// Test infrastructure (tests/test_gpu_evalcb_driver.py builds and runs it); not part of the
// library.  Usage: mock_eval_cb <dir> E k H I S n_tok n_as_full L
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "nvmoe_b200.h"

#define CK(x)                                                                        \
    do {                                                                             \
        cudaError_t e_ = (x);                                                        \
        if (e_ != cudaSuccess) {                                                     \
            std::fprintf(stderr, "%s:%d %s: %s\n", __FILE__, __LINE__, #x,           \
                         cudaGetErrorString(e_));                                    \
            std::exit(3);                                                            \
        }                                                                            \
    } while (0)
#define NV(x)                                                                        \
    do {                                                                             \
        int r_ = (x);                                                                \
        if (r_ != NVMOE_OK) {                                                        \
            std::fprintf(stderr, "%s:%d %s = %d (%s)\n", __FILE__, __LINE__, #x, r_, \
                         nvmoe_last_error());                                        \
            std::exit(4);                                                            \
        }                                                                            \
    } while (0)

enum MockOp { OP_NONE = 0, OP_GET_ROWS = 1, OP_MUL_MAT_ID = 2 };

struct MockTensor {  // the fields of ggml_tensor the callback reads
    int op;
    std::string name;
    void* data;
    int64_t ne[4];
    size_t nb[4];
    MockTensor* src[2];
};

struct LayerCache {  // one layer's slot pool, tables and miss list (moe_cache_probe.cpp:207-250)
    nvmoe_slot_table table;
    nvmoe_miss_list misses;
    nvmoe_expert_pool pool;
    nvmoe_refill_bank banks[6];
};

struct State {
    std::vector<LayerCache> layers;
    int E, S;
    cudaStream_t compute, h2d;
    cudaEvent_t done;
    int status = 0;
    long long refills = 0;
};

static std::vector<char> read_file(const std::string& p, size_t n) {
    std::vector<char> v(n);
    FILE* f = std::fopen(p.c_str(), "rb");
    if (!f || std::fread(v.data(), 1, n, f) != n) {
        std::fprintf(stderr, "cannot read %zu bytes from %s\n", n, p.c_str());
        std::exit(2);
    }
    std::fclose(f);
    return v;
}

static void write_file(const std::string& p, const void* d, size_t n) {
    FILE* f = std::fopen(p.c_str(), "wb");
    if (!f || std::fwrite(d, 1, n, f) != n) std::exit(2);
    std::fclose(f);
}

template <typename T>
static T* dev_alloc(size_t n, int fill = -2) {
    void* p = nullptr;
    CK(cudaMalloc(&p, n * sizeof(T)));
    if (fill != -2) CK(cudaMemset(p, fill == -1 ? 0xff : fill, n * sizeof(T)));
    return static_cast<T*>(p);
}

// The eval callback (moe_cache_probe.cpp:439): ask -> does this node interest us; otherwise run
// the GPU-tier step for the layer named in the node.
static bool eval_cb(MockTensor* t, bool ask, void* ud) {
    State* st = static_cast<State*>(ud);
    const bool mine = t->op == OP_GET_ROWS && t->name.rfind("ffn_moe_weights-", 0) == 0;
    if (ask) return mine;
    if (!mine) return true;
    const int layer = std::atoi(t->name.c_str() + 16);
    LayerCache& L = st->layers[(size_t)layer];
    MockTensor* sel = t->src[1];
    const int k = (int)sel->ne[0], n_tok = (int)sel->ne[1];
    int32_t* ids = static_cast<int32_t*>(sel->data);
    NV(nvmoe_remap(&L.table, ids, (int64_t)sel->nb[1], k, n_tok, 1, ids, (int64_t)sel->nb[1],
                   &L.misses, st->compute));
    int32_t counts[4];
    CK(cudaMemcpyAsync(counts, L.misses.counts, sizeof(counts), cudaMemcpyDeviceToHost,
                       st->compute));
    CK(cudaStreamSynchronize(st->compute));
    if (counts[2] != NVMOE_OK) {  // the reference aborts here; report and stop instead
        st->status = counts[2];
        return false;
    }
    const int n_miss = counts[1];
    if (n_miss > 0) {
        std::vector<int32_t> miss_ids((size_t)n_miss), miss_slots((size_t)n_miss);
        CK(cudaMemcpy(miss_ids.data(), L.misses.miss_ids, 4 * (size_t)n_miss,
                      cudaMemcpyDeviceToHost));
        CK(cudaMemcpy(miss_slots.data(), L.misses.miss_slots, 4 * (size_t)n_miss,
                      cudaMemcpyDeviceToHost));
        // the host tier holds every expert at host slot == expert id
        NV(nvmoe_refill_async(L.banks, 6, miss_slots.data(), miss_ids.data(), n_miss, st->S,
                              st->E, st->h2d, st->compute, st->done));
        st->refills += n_miss;
    }
    return true;
}

int main(int argc, char** argv) {
    if (argc != 10) {
        std::fprintf(stderr, "usage: %s dir E k H I S n_tok n_as_full L\n", argv[0]);
        return 1;
    }
    const std::string dir = argv[1];
    const int E = std::atoi(argv[2]), k = std::atoi(argv[3]), H = std::atoi(argv[4]),
              I = std::atoi(argv[5]), S = std::atoi(argv[6]), n_tok = std::atoi(argv[7]),
              n_as_full = std::atoi(argv[8]), NL = std::atoi(argv[9]);
    State st;
    st.E = E;
    st.S = S;
    int prio_lo = 0, prio_hi = 0;
    CK(cudaDeviceGetStreamPriorityRange(&prio_lo, &prio_hi));
    CK(cudaStreamCreateWithFlags(&st.compute, cudaStreamNonBlocking));
    CK(cudaStreamCreateWithPriority(&st.h2d, cudaStreamNonBlocking, prio_hi));
    CK(cudaEventCreateWithFlags(&st.done, cudaEventDisableTiming));

    // pinned host tier: every expert in the FTW bank layout
    const size_t gu_c = (size_t)2 * I * H / 2, gu_s = (size_t)2 * I * H / 16;
    const size_t dn_c = (size_t)H * I / 2, dn_s = (size_t)H * I / 16;
    const size_t sizes[6] = {gu_c, gu_s, 4, dn_c, dn_s, 4};
    const char* names[6] = {"gu_codes", "gu_scale", "gu_glob", "dn_codes", "dn_scale", "dn_glob"};
    void* host[6];
    for (int b = 0; b < 6; ++b) {
        std::vector<char> v = read_file(dir + "/" + names[b] + ".bin", sizes[b] * (size_t)E);
        CK(cudaHostAlloc(&host[b], sizes[b] * (size_t)E, cudaHostAllocDefault));
        std::memcpy(host[b], v.data(), v.size());
    }
    for (int l = 0; l < NL; ++l) {
        LayerCache L;
        L.table = {dev_alloc<int32_t>((size_t)E, -1), dev_alloc<int32_t>((size_t)S, -1),
                   dev_alloc<uint32_t>((size_t)S, 0), dev_alloc<uint32_t>(1, 0), E, S, 0, 0};
        const int cap = E;
        L.misses = {dev_alloc<int32_t>((size_t)cap), dev_alloc<int32_t>((size_t)cap),
                    dev_alloc<uint8_t>((size_t)cap), dev_alloc<int32_t>((size_t)cap),
                    dev_alloc<int32_t>((size_t)cap), dev_alloc<int32_t>((size_t)cap),
                    dev_alloc<int32_t>(4, 0), cap};
        void* pool[6];
        for (int b = 0; b < 6; ++b) {
            pool[b] = dev_alloc<uint8_t>(sizes[b] * (size_t)S, 0);
            L.banks[b] = {pool[b], host[b], (int64_t)sizes[b], (int64_t)sizes[b], (int64_t)sizes[b]};
        }
        // the reduced ("shrunk") expert tensors: gate = rows [0, I), up = rows [I, 2I)
        auto bank = [&](int c, int s, int g, int64_t rows_off, int K) {
            nvmoe_matrix_bank m;
            m.data = static_cast<uint8_t*>(pool[c]) + rows_off * (K / 2);
            m.slot_stride = (int64_t)sizes[c];
            m.row_stride = K / 2;
            m.scale = static_cast<uint8_t*>(pool[s]) + rows_off * (K / 16);
            m.scale_slot_stride = (int64_t)sizes[s];
            m.scale_row_stride = K / 16;
            m.global_scale = static_cast<const float*>(pool[g]);
            m.global_stride = 1;
            return m;
        };
        L.pool.quant = NVMOE_Q_NVFP4;
        L.pool.hidden = H;
        L.pool.inter = I;
        L.pool.n_slots = S;
        L.pool.gate = bank(0, 1, 2, 0, H);
        L.pool.up = bank(0, 1, 2, I, H);
        L.pool.down = bank(3, 4, 5, 0, I);
        st.layers.push_back(L);
    }

    std::vector<char> xh = read_file(dir + "/x.bin", (size_t)n_tok * H * 2);
    std::vector<char> idh = read_file(dir + "/ids.bin", (size_t)NL * n_tok * k * 4);
    std::vector<char> wh = read_file(dir + "/w.bin", (size_t)NL * n_tok * k * 4);
    uint16_t* x = dev_alloc<uint16_t>((size_t)n_tok * H);
    CK(cudaMemcpy(x, xh.data(), xh.size(), cudaMemcpyHostToDevice));
    uint16_t* y = dev_alloc<uint16_t>((size_t)NL * n_tok * H);
    uint16_t* xin = dev_alloc<uint16_t>((size_t)NL * n_tok * H);  // each layer's input tokens
    uint16_t* hres = dev_alloc<uint16_t>((size_t)n_tok * H);
    CK(cudaMemcpy(xin, x, (size_t)n_tok * H * 2, cudaMemcpyDeviceToDevice));
    std::vector<uint16_t> ones((size_t)H, 0x3F80);  // RMSNorm gamma = 1 (bf16)
    uint16_t* gamma = dev_alloc<uint16_t>((size_t)H);
    CK(cudaMemcpy(gamma, ones.data(), (size_t)H * 2, cudaMemcpyHostToDevice));
    // argsort output [n_as_full, n_tok] per layer; selected_experts is its first k columns
    int32_t* argsort = dev_alloc<int32_t>((size_t)NL * n_tok * n_as_full, -1);
    float* wts = dev_alloc<float>((size_t)NL * n_tok * k);
    for (int l = 0; l < NL; ++l)
        for (int t = 0; t < n_tok; ++t)
            CK(cudaMemcpy(argsort + ((size_t)l * n_tok + t) * n_as_full,
                          idh.data() + ((size_t)l * n_tok + t) * k * 4, (size_t)k * 4,
                          cudaMemcpyHostToDevice));
    CK(cudaMemcpy(wts, wh.data(), wh.size(), cudaMemcpyHostToDevice));
    size_t ws_bytes = nvmoe_moe_ffn_workspace_size(n_tok, k, H, I, S);
    void* ws = dev_alloc<uint8_t>(ws_bytes);
    int32_t* ffn_status = dev_alloc<int32_t>(1, 0);

    for (int l = 0; l < NL; ++l) {
        MockTensor sel{OP_NONE, "ffn_moe_topk-" + std::to_string(l),
                       argsort + (size_t)l * n_tok * n_as_full,
                       {k, n_tok, 1, 1}, {4, (size_t)n_as_full * 4, 0, 0}, {nullptr, nullptr}};
        MockTensor probs{OP_NONE, "ffn_moe_probs-" + std::to_string(l), nullptr, {0}, {0},
                         {nullptr, nullptr}};
        MockTensor weights{OP_GET_ROWS, "ffn_moe_weights-" + std::to_string(l), nullptr,
                           {1, k, n_tok, 1}, {4, 4, (size_t)k * 4, 0}, {&probs, &sel}};
        // the scheduler asks about each node of the layer; only the weights node is claimed
        for (MockTensor* node : {&sel, &probs, &weights}) {
            if (!eval_cb(node, true, &st)) continue;
            if (!eval_cb(node, false, &st)) {
                std::fprintf(stderr, "callback stopped the graph: status %d\n", st.status);
                write_file(dir + "/status.txt", "ERR", 3);
                return 5;
            }
        }
        // mul_mat_id over the reduced tensors: the FFN reads the rewritten ids in place
        nvmoe_ffn_args a;
        std::memset(&a, 0, sizeof(a));
        a.pool = &st.layers[(size_t)l].pool;
        if (l > 0) {  // the chain: RMSNorm(x_{l-1} + y_{l-1})
            nvmoe_router_gate_args g;
            std::memset(&g, 0, sizeof(g));
            g.resid = xin + (size_t)(l - 1) * n_tok * H;
            g.resid_row_stride = H;
            g.delta = y + (size_t)(l - 1) * n_tok * H;
            g.delta_row_stride = H;
            g.resid_out = hres;
            g.resid_out_row_stride = H;
            g.norm_weight = gamma;
            g.eps = 1e-6f;
            g.x_out = xin + (size_t)l * n_tok * H;
            g.x_out_row_stride = H;
            g.n_tok = n_tok;
            g.hidden = H;
            NV(nvmoe_router_gate(&g, st.compute));
        }
        a.x = xin + (size_t)l * n_tok * H;
        a.x_row_stride = H;
        a.slot_ids = static_cast<const int32_t*>(sel.data);
        a.ids_row_stride = n_as_full;
        a.weights = wts + (size_t)l * n_tok * k;
        a.weights_row_stride = k;
        a.top_k = k;
        a.n_tok = n_tok;
        a.y = y + (size_t)l * n_tok * H;
        a.y_row_stride = H;
        a.workspace = ws;
        a.workspace_bytes = ws_bytes;
        a.status = ffn_status;
        NV(nvmoe_moe_ffn(&a, st.compute));
    }
    CK(cudaStreamSynchronize(st.compute));
    int32_t fs = 0;
    CK(cudaMemcpy(&fs, ffn_status, 4, cudaMemcpyDeviceToHost));
    std::vector<uint16_t> yh((size_t)NL * n_tok * H);
    CK(cudaMemcpy(yh.data(), y, yh.size() * 2, cudaMemcpyDeviceToHost));
    std::vector<int32_t> all((size_t)NL * n_tok * n_as_full);
    CK(cudaMemcpy(all.data(), argsort, all.size() * 4, cudaMemcpyDeviceToHost));
    std::vector<int32_t> slots((size_t)NL * n_tok * k);
    for (size_t r = 0; r < (size_t)NL * n_tok; ++r)
        std::memcpy(slots.data() + r * k, all.data() + r * n_as_full, (size_t)k * 4);
    // the columns past the view must be untouched (-1 as filled)
    int untouched = 1;
    for (size_t r = 0; r < (size_t)NL * n_tok; ++r)
        for (int c = k; c < n_as_full; ++c) untouched &= all[r * n_as_full + c] == -1;
    write_file(dir + "/y.bin", yh.data(), yh.size() * 2);
    std::vector<uint16_t> xh2((size_t)NL * n_tok * H);
    CK(cudaMemcpy(xh2.data(), xin, xh2.size() * 2, cudaMemcpyDeviceToHost));
    write_file(dir + "/xin.bin", xh2.data(), xh2.size() * 2);
    write_file(dir + "/slots.bin", slots.data(), slots.size() * 4);
    char msg[128];
    const int m = std::snprintf(msg, sizeof msg, "OK ffn_status=%d refills=%lld untouched=%d", fs,
                                st.refills, untouched);
    write_file(dir + "/status.txt", msg, (size_t)m);
    std::printf("%s\n", msg);
    return 0;
}
