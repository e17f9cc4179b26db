/*
 * nvmoe_b200 — C ABI of the B200 (sm_100a) routed-expert FFN over a VRAM expert-slot cache.
 *
 * Plain pointers and sizes only.  Every entry point returns an int status (NVMOE_OK == 0,
 * negative on error) and never aborts the process.  Device pointers are CUDA device (or
 * managed) addresses; "stream" arguments are cudaStream_t values passed as void*.
 * Kernels that detect bad data on the device (an expert id out of range, more distinct ids
 * than slots) write a status word the host reads back (see nvmoe_miss_list.counts).
 *
 * Reference interfaces these entry points replace (paths inside Waltarb/nvmoe):
 *   - llama.cpp engine: `static bool eval_cb(ggml_tensor*, bool ask, void*)`
 *       scripts/moe_cache_probe.cpp:439-997  (remap, host tier, H2D fill, id rewrite)
 *   - Python engine hook `NvmeOffloadMoeCache` (nvme-moe-bench/nvme_offload_cache.py:441):
 *       ensure_experts :1366, copy_missing :1684, bank_views :954, and the GEMM call
 *       `_expert_gemm(cache, hidden, topk_weights, slot_ids, views, n, alphas, is_prefill)`
 *       :1989-1998 / :2165-2174.
 */
#ifndef NVMOE_B200_H
#define NVMOE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- status codes */
#define NVMOE_OK 0
#define NVMOE_ERR_INVALID_ARG -1    /* bad pointer / size / enum on the host side */
#define NVMOE_ERR_BAD_EXPERT_ID -2  /* an id outside [0, n_expert) reached the remap */
#define NVMOE_ERR_CACHE_OVERFLOW -3 /* more distinct ids in one call than slots */
#define NVMOE_ERR_CUDA -4           /* a CUDA runtime call failed (see nvmoe_last_error) */
#define NVMOE_ERR_WORKSPACE -5      /* workspace pointer null or too small */
#define NVMOE_ERR_UNSUPPORTED -6    /* shape / format combination not built */
#define NVMOE_ERR_HOST_LOAD -7      /* the host-tier loader callback reported a failure */
#define NVMOE_ERR_BAD_SLOT -8       /* a slot id outside [0, n_slots) reached the FFN */
#define NVMOE_ERR_NO_TABLES -9      /* IQ2_XXS grid table not registered */
#define NVMOE_ERR_TIMEOUT -10       /* a bounded wait inside a kernel gave up (status word) */
#define NVMOE_ERR_SCRATCH_LIMIT -11 /* call needs more scratch than nvmoe_moe_ffn_noalloc has */
#define NVMOE_ERR_GROUP_LIMIT -12   /* more token groups than a kernel's group tables hold */

typedef void* nvmoe_stream_t; /* cudaStream_t */
typedef void* nvmoe_event_t;  /* cudaEvent_t  */

/* Weight formats of the slot pool.  NVMOE_Q_NVFP4 is the FTW bank layout of the Python
 * engine (nvme_offload_cache.py:824-835): codes [rows, K/2] u8 with w[2b] in the low nibble
 * of byte b, one E4M3 scale per 16 values [rows, K/16], one fp32 global per slot and matrix.
 * NVMOE_Q_Q2_K / NVMOE_Q_IQ2_XXS are ggml super-blocks of 256 values (84 / 66 bytes).
 * NVMOE_Q_BF16 is the Python engine's bf16 weight banks (the CPU-plumbing layer,
 * nvme_offload_cache.py bank_views); the FFN multiplies them in f16, exact within the f16
 * range. */
enum nvmoe_quant {
    NVMOE_Q_NVFP4 = 0,
    NVMOE_Q_Q2_K = 1,
    NVMOE_Q_IQ2_XXS = 2,
    NVMOE_Q_BF16 = 3, /* plain bf16 rows [rows, K] (2 bytes per value), no scale bank */
};

/* ---------------------------------------------------------------- error text */
/* Text of the last CUDA error seen by this thread inside the library (static storage). */
const char* nvmoe_last_error(void);
/* Library version string, e.g. "nvmoe_b200 0.1.0 sm_100a". */
const char* nvmoe_version(void);

/* ================================================================ R1: router top-k
 * Replaces the router epilogue in front of the expert cache:
 *   llama.cpp softmax -> argsort_top_k -> get_rows -> sum/div  (scripts/test_sched_chain_shrink.cpp:108-121)
 *   GLM sigmoid + e_score_correction_bias -> topk -> gather -> normalize -> * routed_scaling_factor
 *     (nvme-moe-bench/nvme_offload_cache.py:3044-3089)
 * mode NVMOE_ROUTER_SOFTMAX: ids = top_k of logits (ties -> lower expert id);
 *   weights = softmax restricted to the chosen logits (the renormalised softmax top-k),
 *   or the full-softmax probabilities when norm_topk == 0.
 * mode NVMOE_ROUTER_SIGMOID_BIAS: s = sigmoid(logit); ids = top_k of s + bias[e];
 *   weights = s[ids] (/ (sum + 1e-20) when norm_topk) * routed_scaling.
 * Ids come out in descending key order.  n_expert <= 1024, top_k <= 32. */
enum nvmoe_router_mode {
    NVMOE_ROUTER_SOFTMAX = 0,
    NVMOE_ROUTER_SIGMOID_BIAS = 1,
};
int nvmoe_router_topk(const float* logits, int64_t logits_row_stride, int n_tok, int n_expert,
                      int top_k, int mode, const float* bias, int norm_topk, float routed_scaling,
                      int32_t* out_ids, int64_t ids_row_stride, float* out_weights,
                      int64_t weights_row_stride, nvmoe_stream_t stream);

/* ================================================================ in front of R1: router gate
 * The steps in front of the router top-k in a decoder stack, in one launch: the residual add
 * and RMSNorm of the decoder layer and the MoE block's router gate (Qwen4ExpMoE.forward's
 * gate.forward(hidden), nvme-moe-bench/nvme_offload_cache.py:2114).  Per token t:
 *   h[t]      = bf16(resid[t] + delta[t])                    (delta NULL: h = resid)
 *   x[t]      = bf16(gamma * bf16(h * 1/sqrt(mean(h^2) + eps)))   (norm_weight NULL: x = h)
 *   logits[t] = x[t] . gate_weight^T (+ logit_bias)          (fp32 accumulation)
 * resid_out (h) and x_out (x) may be NULL; neither may overlap resid or delta.  gate_weight NULL:
 * only h / x are produced.  H is 1024, 2048 or 4096; rows 16-byte aligned.  As the launch after
 * a decode layer step it waits for that step (programmatic dependent launch) and loads its gate
 * rows while the step finishes; pass nvmoe_decode_args.inputs_after_wait = 1 to the step after
 * it. */
typedef struct nvmoe_router_gate_args {
    const uint16_t* resid; /* bf16 [n_tok, H]                                  */
    int64_t resid_row_stride;
    const uint16_t* delta; /* bf16 [n_tok, H] added to resid, may be NULL      */
    int64_t delta_row_stride;
    uint16_t* resid_out;   /* bf16 [n_tok, H] h, may be NULL                   */
    int64_t resid_out_row_stride;
    const uint16_t* norm_weight; /* bf16 [H] RMSNorm gamma, may be NULL          */
    float eps;
    uint16_t* x_out;       /* bf16 [n_tok, H] x, may be NULL                   */
    int64_t x_out_row_stride;
    const uint16_t* gate_weight; /* bf16 [n_expert, H] router gate, may be NULL  */
    int64_t gate_row_stride;     /* elements                                     */
    const float* logit_bias;     /* fp32 [n_expert] added to the logits, may be NULL */
    float* logits;         /* fp32 [n_tok, n_expert]                           */
    int64_t logits_row_stride;
    int32_t n_tok;
    int32_t hidden;
    int32_t n_expert;
    /* Optional router top-k in the same launch (top_k > 0): once a block of 8 tokens has all its
     * logits, the last CTA to finish on it routes them exactly as nvmoe_router_topk does (mode,
     * bias, norm_topk, routed_scaling alike) into out_ids / out_weights [n_tok, top_k]
     * (contiguous).  tickets: device ints [ceil(n_tok / 8)], zero before the first call; every
     * call leaves them zero again. */
    int32_t top_k;
    int32_t router_mode;
    const float* router_bias;
    int32_t norm_topk;
    float routed_scaling;
    int32_t* out_ids;
    float* out_weights;
    int32_t* tickets;
} nvmoe_router_gate_args;

int nvmoe_router_gate(const nvmoe_router_gate_args* args, nvmoe_stream_t stream);

/* ================================================================ R2/R3/R6: slot remap
 * Device-resident slot tables of one slot pool (one layer in the llama.cpp engine:
 * layer_cache.slot_of_real / real_in_slot / slot_last_used / current_step,
 * scripts/moe_cache_probe.cpp:237-241).  All arrays are device memory owned by the caller. */
typedef struct nvmoe_slot_table {
    int32_t* slot_of_real;    /* [n_expert]   slot holding expert e, -1 = not resident   */
    int32_t* real_in_slot;    /* [cache_size] expert in slot s, -1 = empty               */
    uint32_t* slot_last_used; /* [cache_size] step of the last use of slot s             */
    uint32_t* current_step;   /* [1]          incremented once per remap call            */
    int32_t n_expert;         /* ids are valid in [0, n_expert)                          */
    int32_t cache_size;       /* number of slots                                         */
    int32_t pinned_k;         /* decode calls look for victims in [pinned_k, cache_size) first */
    int32_t id_base;          /* added to every id before the lookup (global pools: layer*E) */
} nvmoe_slot_table;

/* Outputs of one remap call (device memory, capacity >= n_tok*top_k entries each). */
typedef struct nvmoe_miss_list {
    int32_t* unique_ids;  /* distinct ids in first-occurrence order                     */
    int32_t* unique_slot; /* slot of each distinct id after the call                    */
    uint8_t* unique_hit;  /* 1 = the id was resident before the call                    */
    int32_t* miss_ids;    /* ids that were not resident, in first-occurrence order      */
    int32_t* miss_slots;  /* slot chosen for each miss                                  */
    int32_t* evicted_ids; /* previous occupant (as stored: id_base + id), -1 = was empty */
    int32_t* counts;      /* [4]: n_unique, n_miss, status (NVMOE_OK or error), n_ids   */
    int32_t capacity;     /* entries allocated in each list                             */
} nvmoe_miss_list;

/* One remap call == the GPU-tier part of eval_cb (scripts/moe_cache_probe.cpp:627-753,
 * 955-970): distinct ids in first-occurrence order; hits refresh slot_last_used; each miss,
 * in order, takes the first empty slot of [start, cache_size), else the slot with the oldest
 * slot_last_used (ties -> lowest slot) whose occupant is not among this call's ids, where
 * start = pinned_k for decode calls and 0 otherwise, falling back to [0, start); finally every
 * id is rewritten to its slot.  ids are read with a row stride in bytes (ggml nb[1]); out may
 * alias ids.  On a bad id or overflow nothing is modified and counts[2] holds the error. */
int nvmoe_remap(const nvmoe_slot_table* table, const int32_t* ids, int64_t ids_row_stride_bytes,
                int top_k, int n_tok, int is_decode, int32_t* out_slots,
                int64_t out_row_stride_bytes, const nvmoe_miss_list* misses,
                nvmoe_stream_t stream);

/* ================================================================ R8: dequant to memory
 * Bit-exact dequantisation (fp32 out) used by the parity tests and loaders.
 * NVFP4 (FTW banks): out[r, c] = (e2m1(code) * e4m3(scale[r, c/16])) * global  (global may be NULL = 1).
 * Q2_K / IQ2_XXS: ggml block formats, 256 values per block, same operation order as ggml's
 * dequantize_row_* (fp32 products, two roundings for Q2_K: d*sc*q - dmin*m). */
int nvmoe_dequant_nvfp4(const uint8_t* codes, const uint8_t* scales, const float* global_scale,
                        int64_t n_rows, int64_t n_cols, float* out, nvmoe_stream_t stream);
int nvmoe_dequant_q2_k(const void* blocks, int64_t n_blocks, float* out, nvmoe_stream_t stream);
int nvmoe_dequant_iq2_xxs(const void* blocks, int64_t n_blocks, float* out,
                          nvmoe_stream_t stream);

/* Registers the IQ2_XXS codebook (256 entries x 8 magnitudes, bytes) on the current device.
 * The grid is ggml's iq2xxs_grid; callers pass the copy shipped with gguf-py (or ggml). */
int nvmoe_set_iq2xxs_grid(const uint8_t* grid_256x8);

/* ================================================================ R7/R9: routed-expert FFN
 * One quantised matrix bank of a slot pool: slot s of the matrix starts at
 * base + s * slot_stride bytes; its rows are row_stride bytes apart.  For NVFP4 the codes,
 * e4m3 scales and fp32 global are three separate banks (FTW layout); for Q2_K / IQ2_XXS
 * scale/global are NULL. */
typedef struct nvmoe_matrix_bank {
    const void* data;
    int64_t slot_stride; /* bytes between slots                      */
    int64_t row_stride;  /* bytes between rows of one slot           */
    const void* scale;   /* NVFP4: e4m3 [rows, K/16] per slot         */
    int64_t scale_slot_stride;
    int64_t scale_row_stride;
    const float* global_scale; /* NVFP4: [n_slots] fp32 (stride global_stride), may be NULL */
    int64_t global_stride;     /* in floats                                                 */
} nvmoe_matrix_bank;

/* The three matrices of one expert pool: gate [I, H], up [I, H], down [H, I].
 * FTW fused banks (gate_up_packed [S, 2I, H/2]): gate = rows [0, I), up = rows [I, 2I) of the
 * same bank, i.e. up.data = gate.data + I*row_stride with the same slot stride. */
typedef struct nvmoe_expert_pool {
    int32_t quant;  /* enum nvmoe_quant                         */
    int32_t hidden; /* H                                        */
    int32_t inter;  /* I                                        */
    int32_t n_slots;
    nvmoe_matrix_bank gate, up, down;
} nvmoe_expert_pool;

/* Kernel choice of one FFN call (nvmoe_ffn_args.kernel); the configuration the reference reads
 * from NVMOE_* / FREETOKEN_* environment variables travels here, per call, instead.
 *   NVMOE_KERNEL_DEFAULT: nvmoe_moe_ffn runs the mma.sync kernel; nvmoe_moe_ffn_prefill runs the
 *     block-scaled FP4 kernel where the shapes allow it, else the kind::f16 kernel.
 *   NVMOE_KERNEL_MMA: decode FFN on in-register dequantised weights feeding mma.sync.
 *   NVMOE_KERNEL_FP4: block-scaled FP4 tensor-core MMAs (tcgen05 kind::mxf4nvf4) on the NVFP4
 *     banks as stored (decode: NVFP4 pools with H and I multiples of 256, <= 256 tokens; it falls
 *     back to NVMOE_KERNEL_MMA where those do not hold).
 *   NVMOE_KERNEL_F16: prefill on tcgen05 kind::f16 MMAs with the weights dequantised into
 *     tensor memory. */
enum nvmoe_kernel {
    NVMOE_KERNEL_DEFAULT = 0,
    NVMOE_KERNEL_MMA = 1,
    NVMOE_KERNEL_FP4 = 2,
    NVMOE_KERNEL_F16 = 3,
};

/* Arguments of one FFN call.  y[t] = sum_j w[t,j] * down_s( silu(gate_s x[t]) * up_s x[t] ),
 * s = slot_ids[t, j] (a negative slot id is an empty entry: it contributes nothing; ids >= n_slots
 * are reported as NVMOE_ERR_BAD_SLOT); plus, when `shared` is set, the always-on shared expert (slot 0 of that
 * pool) with weight 1, or sigmoid(x[t] . shared_gate) when shared_gate (bf16 [H]) is set
 * (nvme_offload_cache.py:2115-2123).  fp32 accumulation, bf16 in / out. */
typedef struct nvmoe_ffn_args {
    const nvmoe_expert_pool* pool;   /* routed experts                       */
    const nvmoe_expert_pool* shared; /* may be NULL                          */
    const uint16_t* shared_gate;     /* bf16 [H], may be NULL                */
    const uint16_t* x;               /* bf16 [n_tok, H]                      */
    int64_t x_row_stride;            /* elements                             */
    const int32_t* slot_ids;         /* [n_tok, top_k] slot ids              */
    int64_t ids_row_stride;          /* elements                             */
    const float* weights;            /* [n_tok, top_k] combine weights       */
    int64_t weights_row_stride;      /* elements                             */
    int32_t top_k;
    int32_t n_tok;
    uint16_t* y;          /* bf16 [n_tok, H]                                  */
    int64_t y_row_stride; /* elements                                         */
    void* workspace;      /* device scratch, >= nvmoe_moe_ffn_workspace_size  */
    size_t workspace_bytes;
    int32_t* status;      /* optional device int: NVMOE_ERR_BAD_SLOT on a bad slot id */
    int32_t kernel;       /* enum nvmoe_kernel: which kernel runs the call (0 = the default) */
} nvmoe_ffn_args;

size_t nvmoe_moe_ffn_workspace_size(int n_tok, int top_k, int hidden, int inter, int n_slots);
int nvmoe_moe_ffn(const nvmoe_ffn_args* args, nvmoe_stream_t stream);
/* nvmoe_moe_ffn in its two launches, for callers that schedule (or time) them apart:
 * _prepare groups the routed entries by slot into the workspace (token rows, group records);
 * _execute runs the fused expert kernel on that workspace.  Same args for both, in that order
 * on one stream, with nothing in between that writes the workspace.  An addition of this library
 * (the reference's _expert_gemm is one opaque call). */
int nvmoe_moe_ffn_prepare(const nvmoe_ffn_args* args, nvmoe_stream_t stream);
int nvmoe_moe_ffn_execute(const nvmoe_ffn_args* args, nvmoe_stream_t stream);

/* Which kernel nvmoe_moe_ffn takes for these arguments (no launch): NVMOE_FFN_PATH_MMA
 * (in-register dequantisation feeding mma.sync; the default) or NVMOE_FFN_PATH_FP4 (block-scaled
 * FP4 MMAs on the tensor cores, weights fed unchanged from the slot banks, activations as 4
 * NVFP4 residual terms), which runs when args->kernel is NVMOE_KERNEL_FP4 and the pool is NVFP4
 * with H and I multiples of 256.  Negative = the call's error status.  An addition of this
 * library (no counterpart in the reference). */
enum { NVMOE_FFN_PATH_MMA = 0, NVMOE_FFN_PATH_FP4 = 1 };
int nvmoe_moe_ffn_path(const nvmoe_ffn_args* args);

/* Same FFN as nvmoe_moe_ffn, for callers that cannot allocate device memory when they run it
 * (e.g. a llama.cpp eval callback, where every device buffer belongs to ggml's allocator and a
 * cudaMalloc would synchronise the device mid-graph, or a process whose spare VRAM is all given
 * to the slot pool).  No counterpart in the reference: it is an addition of this library.
 * args->workspace / workspace_bytes are ignored: the scratch is one 16 MiB device array built
 * into the library, present on every GPU that loads it until the process exits.  Calls whose
 * nvmoe_moe_ffn_workspace_size exceeds 16 MiB return NVMOE_ERR_SCRATCH_LIMIT.  The first call on
 * a device looks up the array's address (once per device); make it before any stream capture.
 * The address is cached for the process's life and does not survive cudaDeviceReset: do not
 * call this entry point on a device after resetting it.
 * All calls on a device share the array (it keeps the last call's contents; nothing in it needs
 * to start at zero), so calls that overlap on the GPU race: serialise them.  Allocates nothing. */
int nvmoe_moe_ffn_noalloc(const nvmoe_ffn_args* args, nvmoe_stream_t stream);

/* R10 — the same FFN for large batches (prefill, ~1k tokens and up): entries sorted by slot into
 * tiles, each expert's gate/up and down as tcgen05 grouped GEMMs (NVFP4 pools).  Default kernel:
 * block-scaled FP4 MMAs (kind::mxf4nvf4) on the slot banks' codes and scales as stored, the
 * activations as 3 NVFP4 residual terms, tiles of 42 entries (3 x 42 = 126 MMA rows; H a
 * multiple of 512, I of 256 up to 1536); args->kernel == NVMOE_KERNEL_F16 (or other shapes)
 * selects kind::f16 MMAs on weights dequantised into tensor memory, tiles of 128.  Replaces the narrowed-union prefill's
 * _expert_gemm call (nvme_offload_cache.py:1957-2013) and mul_mat_id for n_tokens > 1
 * (moe_cache_probe.cpp:1668-1684).  Same arguments and result as nvmoe_moe_ffn; workspace >=
 * nvmoe_moe_ffn_prefill_workspace_size (the sorted activation images, h and the per-entry
 * outputs: about n_tok*(k+1)*(11H/4+6.5I) bytes on the FP4 path). */
size_t nvmoe_moe_ffn_prefill_workspace_size(int n_tok, int top_k, int hidden, int inter,
                                            int n_slots);
int nvmoe_moe_ffn_prefill(const nvmoe_ffn_args* args, nvmoe_stream_t stream);

/* ================================================================ R4: host tier (SLRU)
 * Segmented LRU of the pinned host tier (nvme_offload_cache.py:333-409;
 * scripts/segmented_host_lru.hpp:85-160): probation queue for first references, protected
 * queue (capacity max(1, floor(capacity*ratio)), first capacity hint wins) for keys touched
 * again; eviction drains probation's LRU end first.  Keys are int64. */
typedef struct nvmoe_slru nvmoe_slru;
nvmoe_slru* nvmoe_slru_create(double protected_ratio);
void nvmoe_slru_destroy(nvmoe_slru* lru);
void nvmoe_slru_set_capacity_hint(nvmoe_slru* lru, int64_t capacity);
void nvmoe_slru_insert_new(nvmoe_slru* lru, int64_t key);
void nvmoe_slru_touch(nvmoe_slru* lru, int64_t key);
int nvmoe_slru_contains(const nvmoe_slru* lru, int64_t key);
int64_t nvmoe_slru_size(const nvmoe_slru* lru);
/* Pops probation's LRU key, else protected's; returns 0 and the key, or -1 when empty. */
int nvmoe_slru_pop_lru(nvmoe_slru* lru, int64_t* key_out);
/* Pops the least recent key not in protect[0..n) (probation first, then protected); when every
 * key is protected falls back to nvmoe_slru_pop_lru (segmented_host_lru.hpp:130-141). */
int nvmoe_slru_pop_lru_excluding(nvmoe_slru* lru, const int64_t* protect, int n_protect,
                                 int64_t* key_out);
void nvmoe_slru_discard(nvmoe_slru* lru, int64_t key);

/* The bounded pinned host tier of one layer (scripts/moe_cache_probe.cpp:636-752 host part):
 * host_slots pinned expert slots in front of the backing store (the reference's NVMe tier),
 * placed by the segmented LRU above with capacity hint host_slots.  One call per layer step,
 * after the GPU remap (nvmoe_remap's miss list read back by the host): GPU hits that are in the
 * host tier are touched; then each GPU miss, in order, is either a host hit (touched; copy it
 * from host_slot_out[m], load_out[m] = 0) or a host miss: a free host slot if any, else the least
 * recent key not among this step's ids (probation first; any key when all are in use), whose
 * expert leaves the host tier; the miss is inserted as new and the caller must fill
 * host_slot_out[m] from the backing store first (load_out[m] = 1).  Host code, no GPU.
 * Returns NVMOE_ERR_CACHE_OVERFLOW when a host miss finds no slot, NVMOE_ERR_BAD_EXPERT_ID for
 * ids outside [0, n_expert). */
typedef struct nvmoe_host_tier nvmoe_host_tier;
nvmoe_host_tier* nvmoe_host_tier_create(int32_t n_expert, int32_t host_slots,
                                        double protected_ratio);
void nvmoe_host_tier_destroy(nvmoe_host_tier* tier);
int nvmoe_host_tier_resolve(nvmoe_host_tier* tier, const int32_t* unique_ids,
                            const uint8_t* unique_hit, int n_unique, const int32_t* miss_ids,
                            int n_miss, int32_t* host_slot_out, uint8_t* load_out);
/* Copies the tier's maps: host slot of each expert [n_expert] (-1: not resident) and expert of
 * each host slot [host_slots] (-1: free).  Either pointer may be NULL. */
int nvmoe_host_tier_tables(const nvmoe_host_tier* tier, int32_t* host_slot_of_id,
                           int32_t* id_in_host_slot);
/* The tier's counts since it was created: misses it served from a host slot (host_hits) and
 * misses that had to be loaded from the backing store (host_misses), over every resolve call.
 * (eval_cb's st->host_hits / st->host_misses, scripts/moe_cache_probe.cpp:727-734.)  Either
 * pointer may be NULL. */
int nvmoe_host_tier_stats(const nvmoe_host_tier* tier, int64_t* host_hits, int64_t* host_misses);

/* ================================================================ (f)3 tail pruning
 * eval_cb's decode-time "two-tier cost-aware expert pruning" (scripts/moe_cache_probe.cpp:
 * 523-625) on the device, between the router top-k and the remap: per token row, picks in
 * neither tier whose share of the row's weight is below nvme_thresh (or whose row already has
 * min_mass of its weight resident), and, with host_thresh > 0, picks only in the host tier below
 * host_thresh, are replaced from the last pick backwards by the row's first slot-resident
 * expert (else the expert of the pool's first occupied slot) with weight 0, keeping at least
 * min_keep picks and min_mass of the weight; the weights are then scaled back to their total.
 * ids / weights [n_tok][top_k] (top_k <= 32) are rewritten in place (row strides in elements).  Like the
 * reference, nothing happens unless nvme_thresh > 0, n_tok * top_k <= 4096 and a slot is
 * occupied; rows with an id outside [0, n_expert) are left as they are.  pruned (device, [2],
 * optional) gains the decode calls' picks pruned from the backing-store tier and from the host
 * tier (eval_cb's decode_pruned_nvme / decode_pruned_host). */
typedef struct nvmoe_prune_args {
    int32_t* ids;
    int64_t ids_row_stride;
    float* weights;
    int64_t weights_row_stride;
    int32_t n_tok;
    int32_t top_k;
    const int32_t* slot_of_real;       /* [n_expert]: slot or -1 (this layer's table)         */
    const int32_t* host_slot_of_real;  /* [n_expert]: host slot or -1; NULL: no host tier       */
    const int32_t* real_in_slot;       /* [cache_size]: expert in each slot or -1              */
    int32_t cache_size;
    int32_t n_expert;
    float nvme_thresh;
    float host_thresh;
    float min_mass;
    int32_t min_keep;
    int32_t is_decode;
    int32_t* pruned;
} nvmoe_prune_args;
int nvmoe_prune_tail(const nvmoe_prune_args* args, nvmoe_stream_t stream);

/* ================================================================ cache counters
 * eval_cb's GPU-tier statistics (scripts/moe_cache_probe.cpp:253-256): distinct ids found in
 * the slot pool or copied in (:662-671), matched callbacks (:995), the same restricted to decode
 * steps, and the bytes copied into the slot pool.  The host tier keeps its own counts
 * (nvmoe_host_tier_stats).  Lives in device memory, zeroed by the caller. */
typedef struct nvmoe_cache_stats {
    int64_t calls;              /* remap calls counted (eval_cb's callback_hits)            */
    int64_t decode_calls;       /* calls with is_decode                                    */
    int64_t gpu_hits;           /* distinct ids already in the slot pool                   */
    int64_t gpu_misses;         /* distinct ids copied into the slot pool                  */
    int64_t decode_gpu_hits;    /* gpu_hits of decode calls                                */
    int64_t decode_gpu_misses;  /* gpu_misses of decode calls                              */
    int64_t refill_bytes;       /* gpu_misses x bytes per expert                           */
    int64_t error_calls;        /* calls whose miss list reported an error (not counted)   */
} nvmoe_cache_stats;

/* Adds one remap call's GPU-tier counts to stats on the device, in stream order after the call
 * that wrote the miss list: counts[0] distinct ids, counts[1] misses, counts[2] status (the
 * nvmoe_miss_list.counts of nvmoe_remap or nvmoe_decode_layer).  No host synchronisation, so it
 * can sit in a captured step.  A call whose status is an error only increments error_calls. */
int nvmoe_cache_stats_add(nvmoe_cache_stats* stats, const int32_t* counts, int is_decode,
                          int64_t bytes_per_expert, nvmoe_stream_t stream);

/* ================================================================ R5: pinned-host refill
 * One bank of an expert row in both tiers: slot s of the device pool starts at
 * dst + s*dst_slot_stride, host slot h of the pinned tier at src + h*src_slot_stride; each
 * copy moves row_bytes.  (gpu_fill_from_host_async, scripts/moe_cache_probe.cpp:377-404;
 * fast_index_copy_multi_jit plan, nvme_offload_cache.py:930-949.) */
typedef struct nvmoe_refill_bank {
    void* dst;
    const void* src;
    int64_t dst_slot_stride;
    int64_t src_slot_stride;
    int64_t row_bytes;
} nvmoe_refill_bank;

/* Issues one cudaMemcpyAsync per (bank, run of consecutive slot pairs) on copy_stream (host
 * arrays gpu_slots / host_slots of length n).  When done is given, `done` is first recorded on
 * compute_stream and waited on by copy_stream (an evicted slot may still be read by FFN work
 * queued there), then recorded on copy_stream after the copies and waited on by
 * compute_stream; a NULL compute_stream is the default stream.  done NULL: no join.
 * Bounds-checked against n_gpu_slots / n_host_slots; host memory must be pinned for the copies
 * to be asynchronous. */
int nvmoe_refill_async(const nvmoe_refill_bank* banks, int n_banks, const int32_t* gpu_slots,
                       const int32_t* host_slots, int n, int32_t n_gpu_slots,
                       int32_t n_host_slots, nvmoe_stream_t copy_stream,
                       nvmoe_stream_t compute_stream, nvmoe_event_t done);

/* Device-driven variant for graph capture: reads n_miss = counts[1], miss_slots[] and the
 * host slot of each miss (host_slot_of_id[miss_ids[m]]) from device memory and copies with
 * an SM kernel from mapped pinned host memory (src pointers must be device-accessible
 * mappings, e.g. cudaHostAlloc'd).  16-byte loads where a bank's bases, strides and row size
 * allow it, 4-byte or byte copies otherwise.  Misses whose host slot is negative (or whose
 * slot is out of range) are skipped and reported as NVMOE_ERR_HOST_LOAD in counts[2]. */
int nvmoe_refill_gather(const nvmoe_refill_bank* banks, int n_banks, const nvmoe_miss_list* misses,
                        const int32_t* host_slot_of_id, int32_t n_gpu_slots,
                        nvmoe_stream_t stream);

/* ================================================================ one decode layer step
 * The whole device-side hot path of one MoE layer in one call, graph-capturable (no host
 * synchronisation): router top-k -> slot remap + miss list -> (optional) refill of the misses
 * from a device-mapped pinned host tier (nvmoe_refill_gather) -> routed-expert FFN + shared
 * expert + combine.  This is eval_cb's GPU-tier work (moe_cache_probe.cpp:439-997) followed by
 * the expert GEMM (_expert_gemm, nvme_offload_cache.py:2142-2184) without the per-layer D2H
 * sync: router, remap and FFN grouping run fused in one kernel.
 * slot_ids / weights receive the rewritten slot ids and combine weights [n_tok, top_k]
 * (contiguous).  ffn.pool / shared / shared_gate / x / y / workspace / status are used;
 * ffn.slot_ids / weights / top_k / n_tok are taken from this struct. */
typedef struct nvmoe_decode_args {
    const float* logits; /* fp32 [n_tok, n_expert]                     */
    int64_t logits_row_stride;
    int32_t router_mode; /* enum nvmoe_router_mode                     */
    const float* router_bias;
    int32_t norm_topk;
    float routed_scaling;
    int32_t top_k;
    int32_t n_tok;
    int32_t is_decode;
    nvmoe_slot_table table;
    nvmoe_miss_list misses;
    int32_t* slot_ids;
    float* weights;
    const nvmoe_refill_bank* refill_banks; /* NULL: no refill (every routed id must be resident) */
    int32_t n_refill_banks;
    const int32_t* host_slot_of_id;
    nvmoe_ffn_args ffn;
    /* 1: the workspace (ffn.workspace) and the miss list of this call are not the ones of the
     * decode step just before it on the stream (a caller running layer after layer alternates
     * two sets), so the step's front kernel writes them while that step's FFN still runs.
     * 0: they are written after it (always correct). */
    int32_t early_outputs;
    /* 1: the logits and token rows are written by the launch just before this call on the
     * stream (nvmoe_router_gate, in a stack whose layers depend on each other), so the step
     * reads them only after waiting for that launch; 0: they were complete before it began. */
    int32_t inputs_after_wait;
    /* Pre-routed steps (logits == NULL): the expert ids [n_tok, top_k] (a negative id is an
     * empty entry, skipped by the remap and the FFN) and their combine weights, e.g. the pairs an
     * expert-parallel rank receives; read after waiting for the launches before this call. */
    const int32_t* routed_ids;
    const float* routed_weights;
    int64_t routed_row_stride; /* elements between rows of routed_ids / routed_weights (0: top_k) */
} nvmoe_decode_args;

int nvmoe_decode_layer(const nvmoe_decode_args* args, nvmoe_stream_t stream);

/* ================================================================ expert parallelism
 * P ranks (one per GPU); rank r owns the routed experts [r*E/P, (r+1)*E/P) under local ids
 * e - r*E/P, and its own copy of the shared expert under local id E/P.  No counterpart in the
 * reference (single GPU); the step is its expert GEMM split across GPUs.  One layer step:
 *   1. nvmoe_ep_dispatch packs this rank's tokens into P send segments of n_tok rows each: a
 *      token goes once to every rank that owns one of its experts (and to this rank for the
 *      shared expert), in token order.  A row holds the token (bf16 [H]), then its local expert
 *      ids on that rank (int32 [k+1]: entry j for routed pick j, -1 where pick j is elsewhere;
 *      entry k the shared expert, on this rank only) and their weights (fp32 [k+1]: the router
 *      weight, 1 or sigmoid(x . shared_gate) for the shared expert), padded to
 *      nvmoe_ep_row_bytes.  Rows past a segment's count have every id -1.  slot_of[t][d] is the
 *      row of token t in segment d (-1: not sent).
 *   2. the caller exchanges the segments (an all-to-all of P equal parts, e.g. NCCL);
 *   3. the owner runs the P*n_tok received rows as one pre-routed step with top_k = k + 1
 *      (nvmoe_decode_layer with routed_ids, or nvmoe_moe_ffn_prefill on its resident pool),
 *      one output row per received row (the weighted sum of that row's local experts);
 *   4. the outputs go back the same way;
 *   5. nvmoe_ep_combine: y[t] = sum over d = 0..P-1 of back[d][slot_of[t][d]], fp32, bf16 out.
 * Every size is fixed by n_tok, so no count crosses to the host and the step can be captured
 * in a CUDA graph. */
size_t nvmoe_ep_row_bytes(int hidden, int top_k);

typedef struct nvmoe_ep_dispatch_args {
    const uint16_t* x;          /* bf16 [n_tok, H] home tokens                          */
    int64_t x_row_stride;       /* elements                                             */
    const int32_t* ids;         /* [n_tok, top_k] global expert ids (contiguous)        */
    const float* weights;       /* [n_tok, top_k] router weights (contiguous)           */
    const uint16_t* shared_gate;/* bf16 [H], may be NULL (shared expert weight 1)       */
    int32_t with_shared;        /* 1: route every token to this rank's shared expert    */
    int32_t n_tok, top_k, hidden, n_expert, world, rank;
    unsigned char* send;        /* [world][n_tok][nvmoe_ep_row_bytes] device bytes      */
    int32_t* slot_of;           /* [n_tok][world]                                       */
    int32_t* status;            /* optional device int: NVMOE_ERR_BAD_EXPERT_ID          */
} nvmoe_ep_dispatch_args;
int nvmoe_ep_dispatch(const nvmoe_ep_dispatch_args* args, nvmoe_stream_t stream);

typedef struct nvmoe_ep_combine_args {
    const uint16_t* back;       /* bf16 [world][n_tok][H] outputs returned by the owners */
    const int32_t* slot_of;     /* [n_tok][world] from nvmoe_ep_dispatch                 */
    int32_t n_tok, hidden, world;
    uint16_t* y;                /* bf16 [n_tok, H]                                      */
    int64_t y_row_stride;
} nvmoe_ep_combine_args;
int nvmoe_ep_combine(const nvmoe_ep_combine_args* args, nvmoe_stream_t stream);

/* ================================================================ diagnostics
 * Block-scaled FP4 tensor-core throughput probe: n_ctas CTAs (at most one per SM) each issue
 * n_iter x 8 tcgen05.mma kind::mxf4nvf4.block16 instructions of the prefill kernel's shape
 * (M 128, N 128, K 64; 2 x 128 x 128 x 64 flops each) on zero operands, back to back; time the
 * launch with events on `stream` for the device's FP4 MMA rate.  status (optional device int)
 * receives NVMOE_ERR_TIMEOUT if the final completion wait gives up.  No counterpart in the
 * reference. */
int nvmoe_probe_fp4_mma(int n_iter, int n_ctas, int32_t* status, nvmoe_stream_t stream);

#ifdef __cplusplus
} /* extern "C" */
#endif

#endif /* NVMOE_B200_H */
