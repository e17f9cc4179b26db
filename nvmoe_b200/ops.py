"""Torch-facing wrappers over the C ABI (device tensors in, device tensors out).

Every function launches the sm_100a kernels of libnvmoe_b200.so on the current CUDA stream and
raises NvmoeError on a non-zero status; nothing here computes on the CPU.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

import torch

from . import _lib
from ._lib import check, lib
from .formats import ExpertWeights, QuantMatrix

_QUANT = {"nvfp4": _lib.NVMOE_Q_NVFP4, "q2_k": _lib.NVMOE_Q_Q2_K, "iq2_xxs": _lib.NVMOE_Q_IQ2_XXS,
          "bf16": _lib.NVMOE_Q_BF16}


_KERNELS = {"default": _lib.NVMOE_KERNEL_DEFAULT, "mma": _lib.NVMOE_KERNEL_MMA,
            "fp4": _lib.NVMOE_KERNEL_FP4, "f16": _lib.NVMOE_KERNEL_F16}


def kernel_choice(kernel: str | None, env_var: str) -> int:
    """nvmoe_ffn_args.kernel for a call: the named kernel ("default", "mma", "fp4", "f16"), or,
    when None, the value of the environment variable env_var (NVMOE_FFN_KERNEL for the decode
    FFN, NVMOE_PREFILL_KERNEL for prefill).  The library itself reads no environment: this
    adapter is the one place the reference's env-style configuration is accepted."""
    import os
    name = kernel if kernel is not None else os.environ.get(env_var, "default")
    try:
        return _KERNELS[name.lower()]
    except KeyError:
        raise ValueError(f"unknown kernel {name!r} (from {env_var if kernel is None else 'argument'});"
                         f" one of {sorted(_KERNELS)}") from None


def _stream(stream=None) -> int:
    s = stream if stream is not None else torch.cuda.current_stream()
    return int(s.cuda_stream)


def _ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def _require_cuda(*ts: torch.Tensor) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("nvmoe_b200 ops take CUDA tensors (there is no CPU path)")


# ------------------------------------------------------------------ R1 router
def router_topk(logits: torch.Tensor, top_k: int, mode: str = "softmax",
                bias: torch.Tensor | None = None, norm_topk: bool = True,
                routed_scaling: float = 1.0, out_ids: torch.Tensor | None = None,
                out_weights: torch.Tensor | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """ids int32 [n, k] and combine weights fp32 [n, k] from fp32 logits [n, E] (written into
    out_ids / out_weights when given: contiguous [n, k])."""
    _require_cuda(logits, bias)
    assert logits.dtype == torch.float32 and logits.dim() == 2 and logits.stride(1) == 1
    n, E = logits.shape
    ids = out_ids if out_ids is not None else torch.empty((n, top_k), dtype=torch.int32,
                                                          device=logits.device)
    w = out_weights if out_weights is not None else torch.empty((n, top_k), dtype=torch.float32,
                                                                device=logits.device)
    assert ids.is_contiguous() and w.is_contiguous()
    m = _lib.NVMOE_ROUTER_SOFTMAX if mode == "softmax" else _lib.NVMOE_ROUTER_SIGMOID_BIAS
    if bias is not None:
        bias = bias.float().contiguous()
    check(lib().nvmoe_router_topk(logits.data_ptr(), logits.stride(0), n, E, top_k, m,
                                  _ptr(bias), int(norm_topk), float(routed_scaling),
                                  ids.data_ptr(), top_k, w.data_ptr(), top_k, _stream()),
          "nvmoe_router_topk")
    return ids, w


# ------------------------------------------------------------------ router gate (in front of R1)
def router_gate_args(resid: torch.Tensor, logits: torch.Tensor | None,
                     gate_weight: torch.Tensor | None, delta: torch.Tensor | None = None,
                     resid_out: torch.Tensor | None = None,
                     norm_weight: torch.Tensor | None = None, eps: float = 1e-6,
                     x_out: torch.Tensor | None = None,
                     logit_bias: torch.Tensor | None = None,
                     route: "tuple | None" = None) -> _lib.RouterGateArgs:
    """C arguments of nvmoe_router_gate over these tensors (bf16 rows, fp32 logits).  route =
    (top_k, out_ids [n, k] int32, out_weights [n, k] fp32, tickets int32 (zeroed),
    mode "softmax" | "sigmoid", router_bias, norm_topk, routed_scaling) fuses the top-k."""
    _require_cuda(resid, logits, gate_weight, delta, resid_out, norm_weight, x_out, logit_bias)
    n, H = resid.shape
    for t in (resid, delta, resid_out, x_out, gate_weight):
        if t is not None:
            assert t.dtype == torch.bfloat16 and t.stride(-1) == 1
    E = 0 if gate_weight is None else gate_weight.shape[0]
    a = _lib.RouterGateArgs(
        resid.data_ptr(), resid.stride(0), _ptr(delta), 0 if delta is None else delta.stride(0),
        _ptr(resid_out), 0 if resid_out is None else resid_out.stride(0), _ptr(norm_weight),
        float(eps), _ptr(x_out), 0 if x_out is None else x_out.stride(0), _ptr(gate_weight),
        0 if gate_weight is None else gate_weight.stride(0), _ptr(logit_bias), _ptr(logits),
        0 if logits is None else logits.stride(0), n, H, E)
    if route is not None:
        k, ids, w, tickets, mode, rbias, norm, scaling = route
        assert ids.is_contiguous() and w.is_contiguous() and tickets.numel() >= (n + 7) // 8
        a.top_k = k
        a.router_mode = (_lib.NVMOE_ROUTER_SOFTMAX if mode == "softmax"
                         else _lib.NVMOE_ROUTER_SIGMOID_BIAS)
        a.router_bias = _ptr(rbias)
        a.norm_topk = int(norm)
        a.routed_scaling = float(scaling)
        a.out_ids, a.out_weights, a.tickets = ids.data_ptr(), w.data_ptr(), tickets.data_ptr()
    return a


def router_gate(resid: torch.Tensor, gate_weight: torch.Tensor | None,
                delta: torch.Tensor | None = None, norm_weight: torch.Tensor | None = None,
                eps: float = 1e-6, logit_bias: torch.Tensor | None = None,
                resid_out: torch.Tensor | None = None, x_out: torch.Tensor | None = None,
                logits: torch.Tensor | None = None):
    """Residual add + RMSNorm + router gate GEMV (nvmoe_router_gate): returns (h, x, logits)
    for bf16 token rows resid [n, H] (+ delta), gate_weight bf16 [E, H]."""
    n, H = resid.shape
    dev = resid.device
    if resid_out is None:
        resid_out = torch.empty((n, H), dtype=torch.bfloat16, device=dev)
    if x_out is None:
        x_out = torch.empty((n, H), dtype=torch.bfloat16, device=dev)
    if logits is None and gate_weight is not None:
        logits = torch.empty((n, gate_weight.shape[0]), dtype=torch.float32, device=dev)
    a = router_gate_args(resid, logits, gate_weight, delta, resid_out, norm_weight, eps, x_out,
                         logit_bias)
    check(lib().nvmoe_router_gate(C.byref(a), _stream()), "nvmoe_router_gate")
    return resid_out, x_out, logits


def residual_add(resid: torch.Tensor, delta: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """out = bf16(resid + delta) (nvmoe_router_gate without norm or gate)."""
    a = router_gate_args(resid, None, None, delta=delta, resid_out=out)
    check(lib().nvmoe_router_gate(C.byref(a), _stream()), "nvmoe_router_gate")
    return out


# ------------------------------------------------------------------ R2/R3/R6 remap
@dataclass
class SlotTableGPU:
    """Device slot tables of one pool (llama.cpp engine layer_cache, moe_cache_probe.cpp:237-241).
    For a global pool (Python engine) pass n_expert = L*E and use id_base = layer*E."""
    n_expert: int
    cache_size: int
    device: torch.device | str = "cuda"
    pinned_k: int = 0
    slot_of_real: torch.Tensor = field(init=False)
    real_in_slot: torch.Tensor = field(init=False)
    last_used: torch.Tensor = field(init=False)
    step: torch.Tensor = field(init=False)

    def __post_init__(self):
        d = self.device
        self.slot_of_real = torch.full((self.n_expert,), -1, dtype=torch.int32, device=d)
        self.real_in_slot = torch.full((self.cache_size,), -1, dtype=torch.int32, device=d)
        self.last_used = torch.zeros((self.cache_size,), dtype=torch.int32, device=d)  # uint32 bits
        self.step = torch.zeros((1,), dtype=torch.int32, device=d)                   # uint32 bits

    def reset(self) -> None:
        self.slot_of_real.fill_(-1)
        self.real_in_slot.fill_(-1)
        self.last_used.zero_()
        self.step.zero_()

    def struct(self, n_expert: int | None = None, id_base: int = 0) -> _lib.SlotTable:
        return _lib.SlotTable(self.slot_of_real.data_ptr(), self.real_in_slot.data_ptr(),
                              self.last_used.data_ptr(), self.step.data_ptr(),
                              self.n_expert if n_expert is None else n_expert, self.cache_size,
                              self.pinned_k, id_base)


@dataclass
class MissListGPU:
    capacity: int
    device: torch.device | str = "cuda"

    def __post_init__(self):
        d, c = self.device, self.capacity
        self.unique_ids = torch.empty(c, dtype=torch.int32, device=d)
        self.unique_slot = torch.empty(c, dtype=torch.int32, device=d)
        self.unique_hit = torch.empty(c, dtype=torch.uint8, device=d)
        self.miss_ids = torch.empty(c, dtype=torch.int32, device=d)
        self.miss_slots = torch.empty(c, dtype=torch.int32, device=d)
        self.evicted_ids = torch.empty(c, dtype=torch.int32, device=d)
        self.counts = torch.zeros(4, dtype=torch.int32, device=d)

    def struct(self) -> _lib.MissList:
        return _lib.MissList(self.unique_ids.data_ptr(), self.unique_slot.data_ptr(),
                             self.unique_hit.data_ptr(), self.miss_ids.data_ptr(),
                             self.miss_slots.data_ptr(), self.evicted_ids.data_ptr(),
                             self.counts.data_ptr(), self.capacity)

    def to_host(self) -> dict:
        c = self.counts.cpu().tolist()
        u, m = c[0], c[1]
        return {
            "n_unique": u, "n_miss": m, "status": c[2],
            "unique_ids": self.unique_ids[:u].cpu().numpy(),
            "unique_slot": self.unique_slot[:u].cpu().numpy(),
            "unique_hit": self.unique_hit[:u].cpu().numpy(),
            "miss_ids": self.miss_ids[:m].cpu().numpy(),
            "miss_slots": self.miss_slots[:m].cpu().numpy(),
            "evicted": self.evicted_ids[:m].cpu().numpy(),
        }


def remap(table: SlotTableGPU, ids: torch.Tensor, is_decode: bool,
          out: torch.Tensor | None = None, misses: MissListGPU | None = None,
          id_base: int = 0, n_expert: int | None = None) -> tuple[torch.Tensor, MissListGPU]:
    """Rewrite expert ids [n_tok, k] (rows may be strided, e.g. a column slice) to slots.
    `out` may be `ids` itself (in-place rewrite, like eval_cb's write-back)."""
    _require_cuda(ids)
    assert ids.dtype == torch.int32 and ids.dim() == 2 and ids.stride(1) == 1
    n_tok, k = ids.shape
    if out is None:
        out = torch.empty((n_tok, k), dtype=torch.int32, device=ids.device)
    cap = max(1, min(n_tok * k, n_expert or table.n_expert))
    if misses is None or misses.capacity < cap:
        misses = MissListGPU(max(cap, n_tok * k), ids.device)
    t = table.struct(n_expert=n_expert, id_base=id_base)
    m = misses.struct()
    check(lib().nvmoe_remap(C.byref(t), ids.data_ptr(), ids.stride(0) * 4, k, n_tok,
                            int(is_decode), out.data_ptr(), out.stride(0) * 4, C.byref(m),
                            _stream()), "nvmoe_remap")
    return out, misses


# ------------------------------------------------------------------ R8 dequant
def dequant_nvfp4(codes: torch.Tensor, scales: torch.Tensor,
                  glob: torch.Tensor | None = None) -> torch.Tensor:
    _require_cuda(codes, scales, glob)
    rows = codes.numel() // codes.shape[-1]
    cols = codes.shape[-1] * 2
    out = torch.empty((*codes.shape[:-1], cols), dtype=torch.float32, device=codes.device)
    check(lib().nvmoe_dequant_nvfp4(codes.contiguous().data_ptr(), scales.contiguous().data_ptr(),
                                    _ptr(glob), rows, cols, out.data_ptr(), _stream()),
          "nvmoe_dequant_nvfp4")
    return out


def dequant_q2_k(blocks: torch.Tensor) -> torch.Tensor:
    _require_cuda(blocks)
    nb = blocks.numel() // 84
    out = torch.empty(nb * 256, dtype=torch.float32, device=blocks.device)
    check(lib().nvmoe_dequant_q2_k(blocks.contiguous().data_ptr(), nb, out.data_ptr(), _stream()),
          "nvmoe_dequant_q2_k")
    return out


_grid_devices: set[int] = set()


def ensure_iq2xxs_grid(device: torch.device | int | None = None) -> None:
    """Registers ggml's IQ2_XXS codebook (from gguf-py) on the device, once."""
    from .formats import iq2xxs_grid
    dev = torch.cuda.current_device() if device is None else torch.device(device).index or 0
    if dev in _grid_devices:
        return
    import numpy as np
    g = np.ascontiguousarray(iq2xxs_grid())
    with torch.cuda.device(dev):
        check(lib().nvmoe_set_iq2xxs_grid(g.ctypes.data), "nvmoe_set_iq2xxs_grid")
    _grid_devices.add(dev)


def dequant_iq2_xxs(blocks: torch.Tensor) -> torch.Tensor:
    _require_cuda(blocks)
    ensure_iq2xxs_grid(blocks.device)
    nb = blocks.numel() // 66
    out = torch.empty(nb * 256, dtype=torch.float32, device=blocks.device)
    check(lib().nvmoe_dequant_iq2_xxs(blocks.contiguous().data_ptr(), nb, out.data_ptr(),
                                      _stream()), "nvmoe_dequant_iq2_xxs")
    return out


# ------------------------------------------------------------------ R7/R9 FFN
def _matrix_bank(m: QuantMatrix, row0: int) -> _lib.MatrixBank:
    d = m.data
    rs = d.stride(1)
    data = d.data_ptr() + row0 * rs
    if m.scale is not None:
        s = m.scale
        scale = s.data_ptr() + row0 * s.stride(1)
        sss, srs = s.stride(0), s.stride(1)
    else:
        scale, sss, srs = None, 0, 0
    glob = None if m.glob is None else m.glob.data_ptr()
    gs = 0 if m.glob is None else m.glob.stride(0)
    return _lib.MatrixBank(data, d.stride(0), rs, scale, sss, srs, glob, gs)


def expert_pool_struct(w: ExpertWeights) -> _lib.ExpertPool:
    """C view of an ExpertWeights pool: gate = rows [0, I) of gate_up, up = rows [I, 2I)."""
    I = w.inter
    return _lib.ExpertPool(_QUANT[w.quant], w.hidden, w.inter, w.n_slots,
                           _matrix_bank(w.gate_up, 0), _matrix_bank(w.gate_up, I),
                           _matrix_bank(w.down, 0))


def ffn_workspace_bytes(n_tok: int, top_k: int, hidden: int, inter: int, n_slots: int) -> int:
    return int(lib().nvmoe_moe_ffn_workspace_size(n_tok, top_k, hidden, inter, n_slots))


class FfnWorkspace:
    """Grow-only device scratch for nvmoe_moe_ffn."""

    def __init__(self, device="cuda"):
        self.device = device
        self.buf = torch.empty(0, dtype=torch.uint8, device=device)

    def get(self, nbytes: int) -> torch.Tensor:
        if self.buf.numel() < nbytes:
            self.buf = torch.zeros(nbytes, dtype=torch.uint8, device=self.device)
        return self.buf


_default_ws: dict[int, FfnWorkspace] = {}


def ffn_path(pool: ExpertWeights, x: torch.Tensor, slot_ids: torch.Tensor,
             weights: torch.Tensor, shared: ExpertWeights | None = None,
             kernel: str | None = None) -> str:
    """Kernel that moe_ffn takes for these arguments: "fp4" (block-scaled FP4 tensor-core
    MMAs) or "mma" (mma.sync on in-register dequantised weights); see nvmoe_moe_ffn_path."""
    _require_cuda(x, slot_ids, weights)
    n, H = x.shape
    k = slot_ids.shape[1]
    ws = _default_ws.setdefault(x.device.index or 0, FfnWorkspace(x.device)).get(
        ffn_workspace_bytes(n, k, pool.hidden, pool.inter, pool.n_slots))
    ps = expert_pool_struct(pool)
    ss = expert_pool_struct(shared) if shared is not None else None
    args = _lib.FfnArgs(
        C.pointer(ps), C.pointer(ss) if ss is not None else None, None, x.data_ptr(),
        x.stride(0), slot_ids.data_ptr(), slot_ids.stride(0), weights.data_ptr(),
        weights.stride(0), k, n, x.data_ptr(), x.stride(0), ws.data_ptr(), ws.numel(), None,
        kernel_choice(kernel, "NVMOE_FFN_KERNEL"))
    rc = lib().nvmoe_moe_ffn_path(C.byref(args))
    check(min(rc, 0), "nvmoe_moe_ffn_path")
    return "fp4" if rc == 1 else "mma"


def moe_ffn(pool: ExpertWeights, x: torch.Tensor, slot_ids: torch.Tensor, weights: torch.Tensor,
            shared: ExpertWeights | None = None, shared_gate: torch.Tensor | None = None,
            out: torch.Tensor | None = None, workspace: FfnWorkspace | None = None,
            status: torch.Tensor | None = None, kernel: str | None = None,
            phase: str = "both") -> torch.Tensor:
    """y = routed-expert FFN over the slot pool (bf16 [n, H]); see nvmoe_moe_ffn.  phase
    "prepare" / "execute" launches one half (nvmoe_moe_ffn_prepare / _execute), "both" the
    whole call."""
    _require_cuda(x, slot_ids, weights)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    assert slot_ids.dtype == torch.int32 and weights.dtype == torch.float32
    n, H = x.shape
    k = slot_ids.shape[1]
    if out is None:
        out = torch.empty((n, H), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        dev = x.device.index or 0
        workspace = _default_ws.setdefault(dev, FfnWorkspace(x.device))
    nbytes = ffn_workspace_bytes(n, k, pool.hidden, pool.inter, pool.n_slots)
    ws = workspace.get(nbytes)
    ps = expert_pool_struct(pool)
    ss = expert_pool_struct(shared) if shared is not None else None
    if shared_gate is not None:
        assert shared_gate.dtype == torch.bfloat16 and shared_gate.is_contiguous()
    args = _lib.FfnArgs(
        C.pointer(ps), C.pointer(ss) if ss is not None else None,
        _ptr(shared_gate), x.data_ptr(), x.stride(0), slot_ids.data_ptr(), slot_ids.stride(0),
        weights.data_ptr(), weights.stride(0), k, n, out.data_ptr(), out.stride(0),
        ws.data_ptr(), ws.numel(), _ptr(status), kernel_choice(kernel, "NVMOE_FFN_KERNEL"))
    fn = {"both": "nvmoe_moe_ffn", "prepare": "nvmoe_moe_ffn_prepare",
          "execute": "nvmoe_moe_ffn_execute"}[phase]
    check(getattr(lib(), fn)(C.byref(args), _stream()), fn)
    return out


def moe_ffn_prefill(pool: ExpertWeights, x: torch.Tensor, slot_ids: torch.Tensor,
                    weights: torch.Tensor, shared: ExpertWeights | None = None,
                    shared_gate: torch.Tensor | None = None, out: torch.Tensor | None = None,
                    workspace: FfnWorkspace | None = None,
                    status: torch.Tensor | None = None, kernel: str | None = None) -> torch.Tensor:
    """The routed-expert FFN for large batches (token-sorted tcgen05 grouped GEMM); same result
    as moe_ffn.  See nvmoe_moe_ffn_prefill."""
    _require_cuda(x, slot_ids, weights)
    assert x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1
    assert slot_ids.dtype == torch.int32 and weights.dtype == torch.float32
    assert slot_ids.stride(1) == 1 and weights.stride(1) == 1
    n, H = x.shape
    k = slot_ids.shape[1]
    if out is None:
        out = torch.empty((n, H), dtype=torch.bfloat16, device=x.device)
    if workspace is None:
        dev = x.device.index or 0
        workspace = _default_ws.setdefault(dev, FfnWorkspace(x.device))
    nbytes = int(lib().nvmoe_moe_ffn_prefill_workspace_size(n, k, pool.hidden, pool.inter,
                                                            pool.n_slots))
    ws = workspace.get(nbytes)
    ps = expert_pool_struct(pool)
    ss = expert_pool_struct(shared) if shared is not None else None
    args = _lib.FfnArgs(
        C.pointer(ps), C.pointer(ss) if ss is not None else None,
        _ptr(shared_gate), x.data_ptr(), x.stride(0), slot_ids.data_ptr(), slot_ids.stride(0),
        weights.data_ptr(), weights.stride(0), k, n, out.data_ptr(), out.stride(0),
        ws.data_ptr(), ws.numel(), _ptr(status), kernel_choice(kernel, "NVMOE_PREFILL_KERNEL"))
    check(lib().nvmoe_moe_ffn_prefill(C.byref(args), _stream()), "nvmoe_moe_ffn_prefill")
    return out


# ------------------------------------------------------------------ (f)3 tail pruning
def prune_tail(ids: torch.Tensor, weights: torch.Tensor, table: "SlotTableGPU",
               nvme_thresh: float, host_thresh: float = 0.0, min_keep: int = 6,
               min_mass: float = 0.95, host_slot_of_real: torch.Tensor | None = None,
               is_decode: bool = True, pruned: torch.Tensor | None = None) -> None:
    """eval_cb's tail pruning (scripts/moe_cache_probe.cpp:523-625) of ids [n, k] (int32) and
    weights [n, k] (fp32) in place, against this layer's slot table (and the host tier's map
    host_slot_of_real [E], if any); see nvmoe_prune_tail.  pruned: int32 [2] device counters."""
    _require_cuda(ids, weights)
    assert ids.dtype == torch.int32 and weights.dtype == torch.float32
    assert ids.stride(1) == 1 and weights.stride(1) == 1 and ids.shape == weights.shape
    n, k = ids.shape
    args = _lib.PruneArgs(ids.data_ptr(), ids.stride(0), weights.data_ptr(), weights.stride(0),
                          n, k, table.slot_of_real.data_ptr(), _ptr(host_slot_of_real),
                          table.real_in_slot.data_ptr(), table.cache_size, table.n_expert,
                          nvme_thresh, host_thresh, min_mass, min_keep, 1 if is_decode else 0,
                          _ptr(pruned))
    check(lib().nvmoe_prune_tail(C.byref(args), _stream()), "nvmoe_prune_tail")


# ------------------------------------------------------------------ cache counters
STATS_FIELDS = tuple(n for n, _ in _lib.CacheStats._fields_)


class CacheStatsGPU:
    """nvmoe_cache_stats in device memory: eval_cb's GPU-tier counters
    (scripts/moe_cache_probe.cpp:253-256, :662-671, :995), accumulated in stream order from the
    miss lists of remap / decode layer calls, without a host round trip."""

    def __init__(self, device="cuda"):
        self.buf = torch.zeros(len(STATS_FIELDS), dtype=torch.int64, device=device)

    def add(self, misses: "MissListGPU", is_decode: bool, bytes_per_expert: int,
            stream=None) -> None:
        check(lib().nvmoe_cache_stats_add(self.buf.data_ptr(), misses.counts.data_ptr(),
                                          1 if is_decode else 0, int(bytes_per_expert),
                                          _stream(stream)), "nvmoe_cache_stats_add")

    def reset(self) -> None:
        self.buf.zero_()

    def read(self) -> dict:
        d = dict(zip(STATS_FIELDS, self.buf.cpu().tolist()))
        refs = d["gpu_hits"] + d["gpu_misses"]
        d["gpu_hit_rate"] = d["gpu_hits"] / refs if refs else 0.0
        return d


# ------------------------------------------------------------------ R5 refill
def refill_banks(gpu: ExpertWeights, host: ExpertWeights) -> list[_lib.RefillBank]:
    """One RefillBank per FTW bank (codes, scales, global) of gate_up and down."""
    out = []
    for g, h in ((gpu.gate_up, host.gate_up), (gpu.down, host.down)):
        for gt, ht in ((g.data, h.data), (g.scale, h.scale), (g.glob, h.glob)):
            if gt is None:
                continue
            rb = gt[0].numel() * gt.element_size()
            out.append(_lib.RefillBank(gt.data_ptr(), ht.data_ptr(), gt.stride(0) * gt.element_size(),
                                       ht.stride(0) * ht.element_size(), rb))
    return out


def refill_async(banks: list[_lib.RefillBank], gpu_slots, host_slots, n_gpu_slots: int,
                 n_host_slots: int, copy_stream: torch.cuda.Stream,
                 compute_stream: torch.cuda.Stream | None, done: torch.cuda.Event | None) -> None:
    import numpy as np
    g = np.ascontiguousarray(gpu_slots, np.int32)
    h = np.ascontiguousarray(host_slots, np.int32)
    arr = (_lib.RefillBank * len(banks))(*banks)
    if done is not None and not done.cuda_event:
        # torch creates the CUDA event on its first record: without one the copy stream and the
        # compute stream would not be joined
        done.record(compute_stream if compute_stream is not None else copy_stream)
    check(lib().nvmoe_refill_async(arr, len(banks), g.ctypes.data, h.ctypes.data, g.size,
                                   n_gpu_slots, n_host_slots, int(copy_stream.cuda_stream),
                                   None if compute_stream is None else int(compute_stream.cuda_stream),
                                   None if done is None else done.cuda_event),
          "nvmoe_refill_async")


def refill_gather(banks: list[_lib.RefillBank], misses: MissListGPU,
                  host_slot_of_id: torch.Tensor, n_gpu_slots: int) -> None:
    arr = (_lib.RefillBank * len(banks))(*banks)
    m = misses.struct()
    check(lib().nvmoe_refill_gather(arr, len(banks), C.byref(m), host_slot_of_id.data_ptr(),
                                    n_gpu_slots, _stream()), "nvmoe_refill_gather")


# ------------------------------------------------------------------ one decode layer step
class DecodeLayerPlan:
    """Pre-built C arguments of nvmoe_decode_layer for one layer (pointers of the layer's slot
    pool, tables, refill banks, workspace and output buffers); call() only patches the per-step
    inputs.  Keeps every ctypes object alive as long as the plan lives."""

    def __init__(self, pool: ExpertWeights, table: SlotTableGPU, misses: MissListGPU,
                 n_tok: int, top_k: int, shared: ExpertWeights | None = None,
                 shared_gate: torch.Tensor | None = None, refill: list | None = None,
                 host_slot_of_id: torch.Tensor | None = None, workspace: FfnWorkspace | None = None,
                 router: str = "softmax", router_bias: torch.Tensor | None = None,
                 norm_topk: bool = True, routed_scaling: float = 1.0, device="cuda",
                 early_outputs: bool = False, kernel: str | None = None,
                 inputs_after_wait: bool = False):
        self.n_tok, self.top_k = n_tok, top_k
        self.pool_s = expert_pool_struct(pool)
        self.shared_s = expert_pool_struct(shared) if shared is not None else None
        self.slot_ids = torch.empty((n_tok, top_k), dtype=torch.int32, device=device)
        self.weights = torch.empty((n_tok, top_k), dtype=torch.float32, device=device)
        self.status = torch.zeros(1, dtype=torch.int32, device=device)
        ws = workspace or FfnWorkspace(device)
        self.ws = ws.get(ffn_workspace_bytes(n_tok, top_k, pool.hidden, pool.inter, pool.n_slots))
        self.refill = (_lib.RefillBank * len(refill))(*refill) if refill else None
        self.table, self.misses, self.host_slot_of_id = table, misses, host_slot_of_id
        self.router_bias, self.shared_gate = router_bias, shared_gate
        a = _lib.DecodeArgs()
        a.router_mode = _lib.NVMOE_ROUTER_SOFTMAX if router == "softmax" else \
            _lib.NVMOE_ROUTER_SIGMOID_BIAS
        a.router_bias = _ptr(router_bias)
        a.norm_topk = int(norm_topk)
        a.routed_scaling = float(routed_scaling)
        a.top_k, a.n_tok, a.is_decode = top_k, n_tok, 1
        a.table = table.struct()
        a.misses = misses.struct()
        a.slot_ids = self.slot_ids.data_ptr()
        a.weights = self.weights.data_ptr()
        if self.refill is not None:
            a.refill_banks = C.cast(self.refill, C.POINTER(_lib.RefillBank))
            a.n_refill_banks = len(refill)
            a.host_slot_of_id = host_slot_of_id.data_ptr()
        a.ffn.pool = C.pointer(self.pool_s)
        if self.shared_s is not None:
            a.ffn.shared = C.pointer(self.shared_s)
        a.ffn.shared_gate = _ptr(shared_gate)
        a.ffn.workspace = self.ws.data_ptr()
        a.ffn.workspace_bytes = self.ws.numel()
        a.ffn.status = self.status.data_ptr()
        a.ffn.kernel = kernel_choice(kernel, "NVMOE_FFN_KERNEL")
        # the caller alternates workspace / miss-list sets between consecutive steps
        a.early_outputs = int(bool(early_outputs))
        a.inputs_after_wait = int(bool(inputs_after_wait))
        self.args = a

    def routed(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
               out: torch.Tensor) -> torch.Tensor:
        """A pre-routed step (no router): expert ids [n_tok, top_k] (negative: empty entry)
        and their weights, rows ids.stride(0) elements apart (the same for both)."""
        assert x.shape[0] == self.n_tok and ids.shape == (self.n_tok, self.top_k)
        assert ids.dtype == torch.int32 and weights.dtype == torch.float32
        assert ids.stride(0) == weights.stride(0) and ids.stride(1) == 1
        a = self.args
        a.logits = None
        a.routed_ids = ids.data_ptr()
        a.routed_weights = weights.data_ptr()
        a.routed_row_stride = ids.stride(0)
        a.ffn.x = x.data_ptr()
        a.ffn.x_row_stride = x.stride(0)
        a.ffn.y = out.data_ptr()
        a.ffn.y_row_stride = out.stride(0)
        check(lib().nvmoe_decode_layer(C.byref(a), _stream()), "nvmoe_decode_layer")
        return out

    def __call__(self, x: torch.Tensor, logits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        assert x.shape[0] == self.n_tok and logits.shape[0] == self.n_tok
        assert x.dtype == torch.bfloat16 and logits.dtype == torch.float32
        a = self.args
        a.logits = logits.data_ptr()
        a.logits_row_stride = logits.stride(0)
        a.routed_ids = a.routed_weights = None
        a.ffn.x = x.data_ptr()
        a.ffn.x_row_stride = x.stride(0)
        a.ffn.y = out.data_ptr()
        a.ffn.y_row_stride = out.stride(0)
        check(lib().nvmoe_decode_layer(C.byref(a), _stream()), "nvmoe_decode_layer")
        return out


# ------------------------------------------------------------------ expert parallelism
def ep_row_bytes(hidden: int, top_k: int) -> int:
    return int(lib().nvmoe_ep_row_bytes(hidden, top_k))


def ep_dispatch(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, n_expert: int,
                world: int, rank: int, send: torch.Tensor, slot_of: torch.Tensor,
                with_shared: bool = True, shared_gate: torch.Tensor | None = None,
                status: torch.Tensor | None = None) -> None:
    """nvmoe_ep_dispatch: this rank's tokens x [n, H] bf16 routed to ids / weights [n, k] into
    send [world, n, ep_row_bytes] u8 and slot_of [n, world] int32."""
    _require_cuda(x, ids, weights, send, slot_of)
    n, H = x.shape
    k = ids.shape[1]
    assert send.dtype == torch.uint8 and send.numel() >= world * n * ep_row_bytes(H, k)
    assert ids.is_contiguous() and weights.is_contiguous() and slot_of.is_contiguous()
    a = _lib.EpDispatchArgs(x.data_ptr(), x.stride(0), ids.data_ptr(), weights.data_ptr(),
                            _ptr(shared_gate), int(with_shared), n, k, H, n_expert, world, rank,
                            send.data_ptr(), slot_of.data_ptr(), _ptr(status))
    check(lib().nvmoe_ep_dispatch(C.byref(a), _stream()), "nvmoe_ep_dispatch")


def ep_combine(back: torch.Tensor, slot_of: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
    """nvmoe_ep_combine: out [n, H] = sum over ranks d of back[d, slot_of[t, d]]."""
    _require_cuda(back, slot_of, out)
    world, n, H = back.shape
    assert back.is_contiguous() and slot_of.is_contiguous()
    a = _lib.EpCombineArgs(back.data_ptr(), slot_of.data_ptr(), n, H, world, out.data_ptr(),
                           out.stride(0))
    check(lib().nvmoe_ep_combine(C.byref(a), _stream()), "nvmoe_ep_combine")
    return out


# ------------------------------------------------------------------ diagnostics
def fp4_mma_tflops(n_iter: int = 4096, reps: int = 3, device=None) -> float:
    """This GPU's block-scaled FP4 MMA rate (TFLOP/s) at the prefill kernel's MMA shape
    (nvmoe_probe_fp4_mma on every SM, CUDA events, best of reps)."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    st = torch.zeros(1, dtype=torch.int32, device=dev)
    flop = float(sms) * n_iter * 8 * 2.0 * 128 * 128 * 64
    check(lib().nvmoe_probe_fp4_mma(64, sms, st.data_ptr(), _stream()), "nvmoe_probe_fp4_mma")
    best = 0.0
    for _ in range(reps):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        check(lib().nvmoe_probe_fp4_mma(n_iter, sms, st.data_ptr(), _stream()),
              "nvmoe_probe_fp4_mma")
        e1.record()
        torch.cuda.synchronize()
        best = max(best, flop / (e0.elapsed_time(e1) / 1e3) / 1e12)
    if int(st.item()) != 0:
        raise _lib.NvmoeError(int(st.item()), "nvmoe_probe_fp4_mma")
    return best
