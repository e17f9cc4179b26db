"""Decode engine over per-layer VRAM slot pools (the llama.cpp engine's layout: one pool of
`cache_size` slots per MoE layer, scripts/moe_cache_probe.cpp:207-250) with a pinned host tier.

One layer step, all on the device and graph-capturable (no host round trip):
    router top-k (R1) -> slot remap + miss list (R2/R3/R6, in place on the ids)
    -> refill of the misses from the pinned host tier by an SM gather (R5)
    -> fused expert FFN + shared expert + combine (R7/R9)
The host tier here holds every expert of a layer at host slot == expert id (the Python engine's
materialised layout, nvme_offload_cache.py:1626-1682), so the miss list alone decides the copies.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass

import numpy as np
import torch

from . import _lib, ops
from .formats import ExpertWeights, QuantMatrix, random_experts


def _slot_view(w: ExpertWeights, start: int, n: int) -> ExpertWeights:
    def sl(m: QuantMatrix) -> QuantMatrix:
        return QuantMatrix(m.quant, m.rows, m.cols, m.data[start:start + n],
                           None if m.scale is None else m.scale[start:start + n],
                           None if m.glob is None else m.glob[start:start + n])
    return ExpertWeights(w.quant, w.hidden, w.inter, sl(w.gate_up), sl(w.down))


def _pin(w: ExpertWeights) -> ExpertWeights:
    def pm(m: QuantMatrix) -> QuantMatrix:
        return QuantMatrix(m.quant, m.rows, m.cols, m.data.pin_memory(),
                           None if m.scale is None else m.scale.pin_memory(),
                           None if m.glob is None else m.glob.pin_memory())
    return ExpertWeights(w.quant, w.hidden, w.inter, pm(w.gate_up), pm(w.down))


def safe_ubatch(cache_size: int, top_k: int) -> int:
    """Largest micro-batch whose distinct routed experts always fit the slot pool, as the
    llama.cpp engine clamps n_ubatch (scripts/moe_cache_probe.cpp:1668-1684):
    min(6, max(1, (cache_size - 4) // top_k))."""
    return min(6, max(1, (cache_size - 4) // top_k))


@dataclass
class StackConfig:
    n_layers: int = 48
    n_experts: int = 512
    top_k: int = 10
    hidden: int = 2048
    inter: int = 512
    cache_size: int = 128
    quant: str = "nvfp4"
    shared_expert: bool = True
    router: str = "softmax"
    pinned_k: int = 0
    # GLM-style routing (router "sigmoid"): top-k of sigmoid(logit) + a per-layer selection
    # bias (set_router_bias), weights renormalised and scaled by routed_scaling
    routed_scaling: float = 1.0
    # tokens per layer call: a batch larger than this runs as consecutive micro-batches, each
    # through every layer, like llama.cpp's n_ubatch (0: the whole batch in one call; the
    # reference's clamp is safe_ubatch(cache_size, top_k))
    ubatch: int = 0


class MoEStack:
    """L MoE layers with device slot pools, slot tables and a shared pinned host tier."""

    def __init__(self, cfg: StackConfig, device="cuda", seed: int = 0,
                 host_tier: ExpertWeights | None = None):
        self.cfg = c = cfg
        self.device = torch.device(device)
        d = self.device
        # host tier: every expert of a layer, pinned, readable by the refill gather (UVA)
        if host_tier is None:
            host_tier = _pin(random_experts(c.quant, c.n_experts, c.hidden, c.inter, seed=seed,
                                            device=d).to("cpu"))
        self.host = host_tier
        # device slot pools: L * cache_size slots in one allocation, one view per layer
        self.pool_all = random_experts(c.quant, c.n_layers * c.cache_size, c.hidden, c.inter,
                                       seed=seed + 1, device=d)
        self.pools = [_slot_view(self.pool_all, l * c.cache_size, c.cache_size)
                      for l in range(c.n_layers)]
        self.shared_all = (random_experts(c.quant, c.n_layers, c.hidden, c.inter, seed=seed + 2,
                                          device=d) if c.shared_expert else None)
        self.shared = ([_slot_view(self.shared_all, l, 1) for l in range(c.n_layers)]
                       if c.shared_expert else [None] * c.n_layers)
        self.tables = [ops.SlotTableGPU(c.n_experts, c.cache_size, d, pinned_k=c.pinned_k)
                       for _ in range(c.n_layers)]
        # two miss lists and FFN workspaces, alternated layer by layer, so that a layer's front
        # kernel can fill its set while the previous layer's FFN still reads the other one
        self.misses_sets = [ops.MissListGPU(c.n_experts, d) for _ in range(2)]
        self.misses = self.misses_sets[(c.n_layers - 1) % 2]  # the last layer's (its misses)
        self.host_slot_of_id = torch.arange(c.n_experts, dtype=torch.int32, device=d)
        self.banks = [ops.refill_banks(p, self.host) for p in self.pools]
        self.ws_sets = [ops.FfnWorkspace(d) for _ in range(2)]
        self._plans: dict[int, list] = {}
        self._chain: dict[int, dict] = {}
        self.gate_w = self.norm_w = self.logit_bias = None
        self.eps = 1e-6
        self.router_bias = None  # [L, E] fp32 selection bias of the sigmoid router

    def set_router_bias(self, bias: np.ndarray) -> None:
        """Per-layer selection bias [L, E] of the sigmoid router (GLM's e_score_correction_bias,
        nvme-moe-bench/nvme_offload_cache.py:3044-3089)."""
        self.router_bias = torch.from_numpy(np.ascontiguousarray(bias, np.float32)).to(self.device)
        self._plans.clear()
        self._chain.clear()

    @property
    def bytes_per_expert(self) -> int:
        return self.pool_all.bytes_per_slot

    def prewarm(self, ranking: np.ndarray) -> None:
        """Fill each layer's slots with its most frequent experts (ranking [L, E], most frequent
        first), like the reference's calibration prewarm (moe_cache_probe.cpp:1335-1466)."""
        c = self.cfg
        cs = torch.cuda.Stream(self.device)
        ev = torch.cuda.Event()
        for l in range(c.n_layers):
            ids = np.asarray(ranking[l][:c.cache_size], np.int32)
            slots = np.arange(len(ids), dtype=np.int32)
            ops.refill_async(self.banks[l], slots, ids, c.cache_size, c.n_experts, cs,
                             torch.cuda.current_stream(self.device), ev)
            t = self.tables[l]
            sor = torch.full((c.n_experts,), -1, dtype=torch.int32)
            sor[torch.from_numpy(ids).long()] = torch.from_numpy(slots)
            ris = torch.full((c.cache_size,), -1, dtype=torch.int32)
            ris[: len(ids)] = torch.from_numpy(ids)
            t.slot_of_real.copy_(sor)
            t.real_in_slot.copy_(ris)
            t.last_used.zero_()
            t.step.zero_()
        torch.cuda.synchronize(self.device)

    def _bias(self, l: int):
        return None if self.router_bias is None else self.router_bias[l]

    def plans(self, n_tok: int) -> list:
        """Per-layer nvmoe_decode_layer argument plans for batches of n_tok tokens."""
        c = self.cfg
        if n_tok not in self._plans:
            # layer l uses set l % 2; with an odd layer count, layer 0 follows the last layer
            # on the same set, so its front writes after its wait
            self._plans[n_tok] = [
                ops.DecodeLayerPlan(self.pools[l], self.tables[l], self.misses_sets[l % 2], n_tok,
                                    c.top_k, shared=self.shared[l], refill=self.banks[l],
                                    host_slot_of_id=self.host_slot_of_id,
                                    workspace=self.ws_sets[l % 2], router=c.router,
                                    router_bias=self._bias(l), routed_scaling=c.routed_scaling,
                                    device=self.device,
                                    early_outputs=not (l == 0 and c.n_layers % 2 == 1))
                for l in range(c.n_layers)]
        return self._plans[n_tok]

    def layer_step(self, l: int, x: torch.Tensor, logits: torch.Tensor,
                   out: torch.Tensor | None = None) -> torch.Tensor:
        """One MoE layer on tokens x [n, H] bf16 with router logits [n, E] fp32: one
        nvmoe_decode_layer call (router, remap, refill gather, FFN)."""
        if out is None:
            out = torch.empty((x.shape[0], self.cfg.hidden), dtype=torch.bfloat16,
                              device=self.device)
        return self.plans(x.shape[0])[l](x, logits, out)

    # ---------------------------------------------------------------- dependent layers
    def init_router(self, logit_bias: np.ndarray | None = None, seed: int = 0,
                    eps: float = 1e-6) -> None:
        """Per-layer router gates for forward_chain: gate weights [L, E, H] bf16 ~ N(0, 1/H)
        (unit-variance logits on RMS-normalised tokens), RMSNorm gammas [L, H] bf16
        ~ 1 + N(0, 0.1), and an optional fp32 logit bias [L, E] (the synthetic routing skew,
        ln p of a Zipf law)."""
        c = self.cfg
        g = torch.Generator().manual_seed(seed)
        self.gate_w = (torch.randn((c.n_layers, c.n_experts, c.hidden), generator=g) /
                       math.sqrt(c.hidden)).to(torch.bfloat16).to(self.device)
        self.norm_w = (1.0 + 0.1 * torch.randn((c.n_layers, c.hidden), generator=g)).to(
            torch.bfloat16).to(self.device)
        self.logit_bias = (None if logit_bias is None else
                           torch.from_numpy(np.ascontiguousarray(logit_bias, np.float32)).to(
                               self.device))
        self.eps = eps
        self._chain.clear()

    def chain_buffers(self, n_tok: int) -> dict:
        """Device buffers and prebuilt C arguments of forward_chain for batches of n_tok: per
        layer the residual h (h[l] enters layer l, l >= 1), the normalised tokens xn, the
        logits and the MoE output y."""
        if self.gate_w is None:
            raise RuntimeError("forward_chain needs init_router() first")
        if n_tok in self._chain:
            return self._chain[n_tok]
        c, d = self.cfg, self.device
        L, H, E = c.n_layers, c.hidden, c.n_experts
        b = {"h": torch.empty((L, n_tok, H), dtype=torch.bfloat16, device=d),
             "xn": torch.empty((L, n_tok, H), dtype=torch.bfloat16, device=d),
             "logits": torch.empty((L, n_tok, E), dtype=torch.float32, device=d),
             "y": torch.empty((L, n_tok, H), dtype=torch.bfloat16, device=d),
             # the router's picks, written by the gate launch itself (fused top-k)
             "ids": torch.empty((L, n_tok, c.top_k), dtype=torch.int32, device=d),
             "w": torch.empty((L, n_tok, c.top_k), dtype=torch.float32, device=d),
             "tickets": torch.zeros(((n_tok + 7) // 8,), dtype=torch.int32, device=d)}
        # Routing: above one token block (8 tokens) the gate launch routes its blocks in
        # parallel (fused top-k, last CTA per block); up to 8 tokens the decode step's front
        # kernel routes them (a warp per token, overlapped with its table loads), which measured
        # faster than the gate launch's extra serial tail.
        b["route_in_gate"] = n_tok > 8
        b["plans"] = [
            ops.DecodeLayerPlan(self.pools[l], self.tables[l], self.misses_sets[l % 2], n_tok,
                                c.top_k, shared=self.shared[l], refill=self.banks[l],
                                host_slot_of_id=self.host_slot_of_id,
                                workspace=self.ws_sets[l % 2], router=c.router,
                                router_bias=self._bias(l), routed_scaling=c.routed_scaling,
                                device=d, early_outputs=False, inputs_after_wait=True)
            for l in range(L)]
        gates = []
        for l in range(L):
            # layers 0 and 1 read the caller's x (patched per call)
            resid = b["h"][l - 1] if l >= 2 else b["xn"][0]
            gates.append(ops.router_gate_args(
                resid, b["logits"][l], self.gate_w[l],
                delta=b["y"][l - 1] if l >= 1 else None,
                resid_out=b["h"][l] if l >= 1 else None, norm_weight=self.norm_w[l],
                eps=self.eps, x_out=b["xn"][l],
                logit_bias=None if self.logit_bias is None else self.logit_bias[l],
                route=(c.top_k, b["ids"][l], b["w"][l], b["tickets"], c.router, self._bias(l),
                       True, c.routed_scaling) if b["route_in_gate"] else None))
        b["gates"] = gates
        self._chain[n_tok] = b
        return b

    def forward_chain(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """L MoE layers whose inputs depend on each other, on tokens x [n, H] bf16:
            h_0 = x;  per layer l: h_l = h_{l-1} + y_{l-1} (l >= 1), xn_l = RMSNorm_l(h_l),
            logits_l = xn_l . gate_l^T + bias_l, y_l = MoE_l(xn_l) (router top-k, slot remap,
            refill, expert FFN, shared expert);  out = h_{L-1} + y_{L-1}.
        Per layer two calls: nvmoe_router_gate (which also routes batches above 8 tokens: fused
        top-k), then nvmoe_decode_layer (routing smaller batches itself), which waits for it."""
        n = x.shape[0]
        b = self.chain_buffers(n)
        L = self.cfg.n_layers
        lib = _lib.lib()
        s = ops._stream()
        for l in range(L):
            ga = b["gates"][l]
            if l == 0:
                ga.resid, ga.resid_row_stride = x.data_ptr(), x.stride(0)
            elif l == 1:
                ga.resid, ga.resid_row_stride = x.data_ptr(), x.stride(0)
            else:
                ga.resid = b["h"][l - 1].data_ptr()
            _lib.check(lib.nvmoe_router_gate(C.byref(ga), s), "nvmoe_router_gate")
            if b["route_in_gate"]:
                b["plans"][l].routed(b["xn"][l], b["ids"][l], b["w"][l], b["y"][l])
            else:
                b["plans"][l](b["xn"][l], b["logits"][l], b["y"][l])
        fin = ops.router_gate_args(x if L == 1 else b["h"][L - 1], None, None,
                                   delta=b["y"][L - 1], resid_out=out)
        _lib.check(lib.nvmoe_router_gate(C.byref(fin), s), "nvmoe_router_gate")
        return out

    def ubatches(self, n_tok: int) -> list[tuple[int, int]]:
        """[start, end) token ranges of the micro-batches a batch of n_tok runs as."""
        u = self.cfg.ubatch if self.cfg.ubatch > 0 else n_tok
        return [(a, min(a + u, n_tok)) for a in range(0, n_tok, u)]

    def forward(self, x: torch.Tensor, logits: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """All layers on the same token batch: logits [L, n, E], out [L, n, H].  With
        cfg.ubatch set, each micro-batch runs through every layer before the next one starts
        (the order llama.cpp decodes a batch split into ubatches)."""
        for a, b in self.ubatches(x.shape[0]):
            plans = self.plans(b - a)
            for l in range(self.cfg.n_layers):
                plans[l](x[a:b], logits[l, a:b], out[l, a:b])
        return out
