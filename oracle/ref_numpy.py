"""numpy restatement of the hot path's floating-point rows (test infrastructure only).

R1 router top-k, R8 dequant (NVFP4 FTW banks, Q2_K, IQ2_XXS), R7/R9 FFN in fp32.
Every function cites the reference behaviour it follows.
"""
from __future__ import annotations

import numpy as np

# ---------------------------------------------------------------- R1 router
def router_topk_softmax(logits: np.ndarray, k: int, norm_topk: bool = True,
                        scaling: float = 1.0):
    """softmax -> top-k -> (renormalise) (llama.cpp build_moe_ffn as exercised by
    scripts/test_sched_chain_shrink.cpp:108-121; Qwen norm_topk_prob).

    Selection uses the logits (softmax is monotone): descending, ties -> lower id.
    Weights: exp(l_j - l_max) summed in pick order, divided by that sum (or by the full
    softmax denominator when norm_topk is False), times `scaling`; fp32 throughout."""
    logits = np.asarray(logits, dtype=np.float32)
    n, E = logits.shape
    key = np.where(np.isnan(logits), -np.inf, logits)
    # lexsort: primary key descending, secondary expert id ascending
    order = np.lexsort((np.broadcast_to(np.arange(E), (n, E)), -key), axis=1)[:, :k]
    ids = order.astype(np.int32)
    sel = np.take_along_axis(logits, order, axis=1)
    m = sel[:, :1]
    w = np.exp((sel - m).astype(np.float32)).astype(np.float32)
    s = np.zeros((n,), np.float32)
    for j in range(k):
        s = (s + w[:, j]).astype(np.float32)
    if norm_topk:
        denom = s
    else:
        full = np.where(np.isnan(logits), 0.0, np.exp((logits - m).astype(np.float32)))
        denom = full.astype(np.float32).sum(axis=1, dtype=np.float32)
    out = (w / denom[:, None]).astype(np.float32) * np.float32(scaling)
    return ids, out.astype(np.float32)


def router_topk_sigmoid_bias(logits: np.ndarray, k: int, bias: np.ndarray | None,
                             norm_topk: bool = True, scaling: float = 1.0):
    """GLM router (nvme-moe-bench/nvme_offload_cache.py:3044-3089): scores = sigmoid(logits);
    choice = scores + e_score_correction_bias; ids = topk(choice); weights = scores[ids]
    / (sum + 1e-20) if norm_topk; * routed_scaling_factor."""
    logits = np.asarray(logits, dtype=np.float32)
    n, E = logits.shape
    s = (np.float32(1.0) / (np.float32(1.0) + np.exp(-logits))).astype(np.float32)
    c = s + (np.asarray(bias, np.float32) if bias is not None else np.float32(0))
    c = np.where(np.isnan(c), -np.inf, c).astype(np.float32)
    order = np.lexsort((np.broadcast_to(np.arange(E), (n, E)), -c), axis=1)[:, :k]
    ids = order.astype(np.int32)
    w = np.take_along_axis(s, order, axis=1).astype(np.float32)
    tot = np.zeros((n,), np.float32)
    for j in range(k):
        tot = (tot + w[:, j]).astype(np.float32)
    if norm_topk:
        w = (w / (tot[:, None] + np.float32(1e-20))).astype(np.float32)
    return ids, (w * np.float32(scaling)).astype(np.float32), c


# ---------------------------------------------------------------- R8 dequant
# code 0x8 (negative zero in E2M1) decodes to +0, as ggml's kvalue table does
_E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                  0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def e4m3fn_to_f32(b: np.ndarray) -> np.ndarray:
    """float8_e4m3fn bits -> fp32 (bias 7, subnormals m*2^-9, 0x7F/0xFF = NaN)."""
    b = np.asarray(b, dtype=np.uint8)
    s = (b >> 7).astype(np.int32)
    e = ((b >> 3) & 0xF).astype(np.int32)
    m = (b & 7).astype(np.float32)
    v = np.where(e == 0, m * np.float32(2.0 ** -9),
                 (np.float32(1.0) + m / np.float32(8.0)) * np.exp2((e - 7).astype(np.float32)))
    v = np.where((e == 15) & (m == 7), np.float32(np.nan), v)
    return np.where(s == 1, -v, v).astype(np.float32)


def dequant_nvfp4(codes: np.ndarray, scales: np.ndarray, global_scale=None) -> np.ndarray:
    """FTW NVFP4 bank rows (scripts/convert_ftw_to_gguf.py:46-58; nvme_offload_cache.py:824-835):
    codes [..., K/2] u8 with w[2b] in the low nibble of byte b; scales [..., K/16] e4m3fn;
    value = (e2m1 * e4m3) * global, fp32 (the first product is exact)."""
    codes = np.asarray(codes, dtype=np.uint8)
    lo = _E2M1[codes & 0xF]
    hi = _E2M1[codes >> 4]
    vals = np.stack([lo, hi], axis=-1).reshape(*codes.shape[:-1], codes.shape[-1] * 2)
    sc = np.repeat(e4m3fn_to_f32(scales), 16, axis=-1)
    out = (vals * sc).astype(np.float32)
    if global_scale is not None:
        out = (out * np.float32(global_scale)).astype(np.float32)
    return out


def dequant_nvfp4_torch(codes, scales, global_scale=None):
    """dequant_nvfp4 restated in torch CPU tensor ops (vectorised and multi-threaded), for the
    parity tests at full layer sizes (512 experts x 1.5 M values).  Same values and the same
    operation order, (e2m1 * e4m3) * global in fp32; a CPU test holds it to dequant_nvfp4 bit
    for bit.  Returns a float32 torch tensor."""
    import torch
    c = torch.as_tensor(codes, dtype=torch.uint8)
    tab = torch.from_numpy(_E2M1)
    lo = tab[(c & 0xF).long()]
    hi = tab[(c >> 4).long()]
    vals = torch.stack([lo, hi], dim=-1).reshape(*c.shape[:-1], c.shape[-1] * 2)
    sc = torch.as_tensor(scales, dtype=torch.uint8).contiguous().view(torch.float8_e4m3fn)
    out = vals * sc.float().repeat_interleave(16, dim=-1)
    if global_scale is not None:
        out = out * torch.tensor(np.float32(global_scale))
    return out


def dequant_q2_k(blocks: np.ndarray) -> np.ndarray:
    """ggml block_q2_K (84 B / 256 values): y = (d*sc)*q - (dmin*m), fp32 with a rounding after
    every operation, value e -> qs[32*(e//128) + e%32] >> 2*((e%128)//32)."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 84)
    nb = b.shape[0]
    sc = b[:, :16]
    qs = b[:, 16:80]
    d = b[:, 80:82].copy().view(np.float16).astype(np.float32).reshape(nb, 1)
    dmin = b[:, 82:84].copy().view(np.float16).astype(np.float32).reshape(nb, 1)
    e = np.arange(256)
    q = (qs[:, 32 * (e // 128) + e % 32] >> (2 * ((e % 128) // 32)).astype(np.uint8)) & 3
    sub = e // 16
    dl = (d * (sc[:, sub] & 0xF).astype(np.float32)).astype(np.float32)
    ml = (dmin * (sc[:, sub] >> 4).astype(np.float32)).astype(np.float32)
    return ((dl * q.astype(np.float32)).astype(np.float32) - ml).astype(np.float32).reshape(-1)


def ksigns() -> np.ndarray:
    """ggml ksigns_iq2xs: 7-bit index with its parity bit as bit 7."""
    i = np.arange(128, dtype=np.uint32)
    par = np.array([bin(v).count("1") & 1 for v in range(128)], dtype=np.uint32)
    return (i | (par << 7)).astype(np.uint8)


def dequant_iq2_xxs(blocks: np.ndarray, grid: np.ndarray) -> np.ndarray:
    """ggml block_iq2_xxs (66 B / 256 values): per 32 values aux0 = 4 codebook indices,
    aux1 = 4 x 7-bit sign indices | scale << 28; db = (d*(0.5+s))*0.25;
    y = (db * grid[idx][i]) * sign."""
    b = np.asarray(blocks, dtype=np.uint8).reshape(-1, 66)
    nb = b.shape[0]
    d = b[:, :2].copy().view(np.float16).astype(np.float32).reshape(nb, 1, 1, 1)
    q = b[:, 2:].copy().view(np.uint32).reshape(nb, 8, 2)
    aux0, aux1 = q[..., 0], q[..., 1]
    db = ((d * (np.float32(0.5) + (aux1 >> 28).astype(np.float32)).reshape(nb, 8, 1, 1))
          .astype(np.float32) * np.float32(0.25)).astype(np.float32)
    idx = aux0.copy().view(np.uint8).reshape(nb, 8, 4)
    mag = np.asarray(grid, np.float32).reshape(256, 8)[idx]  # nb,8,4,8
    sidx = (aux1.reshape(nb, 8, 1) >> np.array([0, 7, 14, 21], np.uint32)) & 127
    sb = ksigns()[sidx]  # nb,8,4
    bits = (sb[..., None] >> np.arange(8, dtype=np.uint8)) & 1
    sign = np.where(bits == 1, np.float32(-1), np.float32(1))
    return ((db * mag).astype(np.float32) * sign).astype(np.float32).reshape(-1)


# ---------------------------------------------------------------- R7 / R9 FFN
def bf16_to_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x, dtype=np.uint16)
    return (x.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """round-to-nearest-even fp32 -> bf16 bits (NaN kept quiet)."""
    x = np.asarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    return np.where(np.isnan(x), np.uint16(0x7FC0), r).astype(np.uint16)


def silu(g: np.ndarray) -> np.ndarray:
    g = g.astype(np.float32)
    return (g / (np.float32(1.0) + np.exp(-g))).astype(np.float32)


def moe_ffn(x_bf16: np.ndarray, slot_ids: np.ndarray, weights: np.ndarray, gate_w, up_w, down_w,
            shared=None, shared_gate_bf16: np.ndarray | None = None) -> np.ndarray:
    """y[t] = sum_j w[t,j] * down_s(silu(gate_s x[t]) * up_s x[t]) (+ shared expert with weight 1
    or sigmoid(x . g_shared)), fp32 accumulation, returns fp32 (caller rounds to bf16).

    gate_w / up_w / down_w: callables slot -> dense fp32 [I,H] / [I,H] / [H,I] (dequantised with
    the functions above); shared: (gate [I,H], up [I,H], down [H,I]) fp32 or None.
    Mirrors _expert_gemm's contract (nvme_offload_cache.py:1989-1998, 2165-2174) and
    Qwen4ExpMoE.forward's shared-expert combine (:2114-2123)."""
    x = bf16_to_f32(x_bf16)
    n, H = x.shape
    y = np.zeros((n, H), np.float32)
    ids = np.asarray(slot_ids)
    w = np.asarray(weights, np.float32)
    for s in np.unique(ids):
        toks, js = np.nonzero(ids == s)
        G, U, D = gate_w(int(s)), up_w(int(s)), down_w(int(s))
        xs = x[toks]
        h = (silu(xs @ G.T) * (xs @ U.T)).astype(np.float32)
        out = (h @ D.T).astype(np.float32)
        y[toks] += w[toks, js][:, None] * out
    if shared is not None:
        G, U, D = shared
        h = (silu(x @ G.T) * (x @ U.T)).astype(np.float32)
        out = (h @ D.T).astype(np.float32)
        if shared_gate_bf16 is not None:
            gv = x @ bf16_to_f32(shared_gate_bf16)
            out = out * (np.float32(1) / (np.float32(1) + np.exp(-gv)))[:, None]
        y += out
    return y


# ---------------------------------------------------------------- in front of R1: router gate
def residual_add_bf16(a_bits: np.ndarray, b_bits: np.ndarray | None) -> np.ndarray:
    """h = bf16(a + b) for bf16 rows (fp32 add, one round-to-nearest-even): the decoder layer's
    residual add in front of the MoE block."""
    a = bf16_to_f32(a_bits)
    if b_bits is None:
        return np.asarray(a_bits, np.uint16)
    return f32_to_bf16((a + bf16_to_f32(b_bits)).astype(np.float32))


def rmsnorm_bf16(h_bits: np.ndarray, gamma_bits: np.ndarray | None, eps: float) -> np.ndarray:
    """x = bf16(gamma * bf16(h * (1 / sqrt(mean(h^2) + eps)))) per row, fp32 statistics (the
    RMSNorm of the decoder layer whose output feeds Qwen4ExpMoE.forward's gate.forward,
    nvme-moe-bench/nvme_offload_cache.py:2114); gamma None: x = h."""
    if gamma_bits is None:
        return np.asarray(h_bits, np.uint16)
    h = bf16_to_f32(h_bits)
    H = h.shape[-1]
    var = (np.sum(h.astype(np.float64) ** 2, axis=-1) / H).astype(np.float32)
    inv = (np.float32(1.0) / np.sqrt((var + np.float32(eps)).astype(np.float32))).astype(np.float32)
    n = f32_to_bf16((h * inv[..., None]).astype(np.float32))
    return f32_to_bf16((bf16_to_f32(gamma_bits) * bf16_to_f32(n)).astype(np.float32))


def router_gate_logits(x_bits: np.ndarray, w_bits: np.ndarray,
                       bias: np.ndarray | None = None) -> np.ndarray:
    """logits = x . W^T (+ bias): the MoE block's router gate (gate.forward,
    nvme_offload_cache.py:2114), accumulated in float64 and returned as fp32."""
    lg = bf16_to_f32(x_bits).astype(np.float64) @ bf16_to_f32(w_bits).astype(np.float64).T
    if bias is not None:
        lg = lg + np.asarray(bias, np.float64)
    return lg.astype(np.float32)


def prune_tail(ids, w, slot_of_real, host_slot_of_real, real_in_slot, nvme_thresh, host_thresh,
               min_keep, min_mass, is_decode=True):
    """eval_cb's two-tier cost-aware tail pruning (scripts/moe_cache_probe.cpp:523-625) of ids /
    weights [n, k], restated with fp32 scalar arithmetic in the reference's order.  Returns the
    new ids, weights and the (backing-store, host) picks pruned in decode calls.  host_slot_of_real
    None: no host tier."""
    f32 = np.float32
    ids = np.array(ids, np.int32, copy=True)
    w = np.array(w, np.float32, copy=True)
    n, k = ids.shape
    pn = ph = 0
    if not f32(nvme_thresh) > 0 or n * k > 4096:
        return ids, w, 0, 0
    occupied = [int(r) for r in real_in_slot if r != -1]
    if not occupied:
        return ids, w, 0, 0
    resident_real = occupied[0]
    in_gpu = lambda r: slot_of_real[r] != -1  # noqa: E731
    in_host = lambda r: host_slot_of_real is not None and host_slot_of_real[r] != -1  # noqa: E731
    for row in range(n):
        if ((ids[row] < 0) | (ids[row] >= len(slot_of_real))).any():
            continue
        total = f32(0)
        for i in range(k):
            total = f32(total + w[row, i])
        if not total > f32(1e-6):
            continue
        gpu_res, in_mem = -1, f32(0)
        for i in range(k):
            r = ids[row, i]
            if in_gpu(r) and gpu_res == -1:
                gpu_res = int(r)
            if in_gpu(r) or in_host(r):
                in_mem = f32(in_mem + f32(w[row, i] / total))
        alias = gpu_res if gpu_res != -1 else resident_real
        remaining, kept, modified = f32(1), k, False
        for j in range(k - 1, -1, -1):
            if kept <= min_keep:
                break
            r = ids[row, j]
            if in_gpu(r):
                continue
            rel = f32(w[row, j] / total)
            if in_host(r):
                if f32(host_thresh) > 0 and rel < f32(host_thresh) and \
                        f32(remaining - rel) >= f32(min_mass):
                    w[row, j], ids[row, j] = 0, alias
                    remaining, kept, modified = f32(remaining - rel), kept - 1, True
                    ph += 1 if is_decode else 0
                continue
            should = rel < f32(nvme_thresh) or in_mem >= f32(min_mass)
            if should and f32(remaining - rel) >= f32(min_mass):
                w[row, j], ids[row, j] = 0, alias
                remaining, kept, modified = f32(remaining - rel), kept - 1, True
                pn += 1 if is_decode else 0
        if modified:
            new_total = f32(0)
            for i in range(k):
                new_total = f32(new_total + w[row, i])
            if new_total > f32(1e-6):
                fac = f32(total / new_total)
                for i in range(k):
                    w[row, i] = f32(w[row, i] * fac)
    return ids, w, pn, ph
