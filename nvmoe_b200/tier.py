"""The bounded pinned host tier (the llama.cpp engine's middle tier) on the hot path.

HostTier owns one layer's native host tier (nvmoe_host_tier_*: slot maps and the segmented LRU of
scripts/segmented_host_lru.hpp, placed as eval_cb does, scripts/moe_cache_probe.cpp:636-752).

BoundedTierStack is a decode stack of dependent layers whose host tier holds fewer experts than
the model.  Each layer step is eval_cb's flow: the GPU remap's miss list comes back to the host
(one small read per layer step, as in the reference), the host tier places the misses, experts
missing from it are loaded from the backing store into their pinned host slots, and the misses
are copied into their GPU slots by cudaMemcpyAsync on a side stream (nvmoe_refill_async) that
the FFN waits for through an event.  The backing store stands in for the reference's io_uring
NVMe tier, which is outside this path: it is pageable host memory, read with a memcpy.
"""
from __future__ import annotations

import ctypes as C
import dataclasses

import numpy as np
import torch

from . import _lib, ops
from ._lib import check, lib
from .formats import ExpertWeights, QuantMatrix


class HostTier:
    def __init__(self, n_expert: int, host_slots: int, protected_ratio: float = 0.8):
        self.n_expert, self.host_slots = n_expert, host_slots
        self.h = lib().nvmoe_host_tier_create(n_expert, host_slots, protected_ratio)
        if not self.h:
            raise ValueError("nvmoe_host_tier_create rejected its arguments")

    def __del__(self):
        h, self.h = getattr(self, "h", None), None
        if h and _lib._lib is not None:  # (the library may be gone at interpreter exit)
            _lib._lib.nvmoe_host_tier_destroy(h)

    def resolve(self, unique_ids, unique_hit, miss_ids):
        """(host slot of each miss, 1 where that slot must first be loaded)."""
        u = np.ascontiguousarray(unique_ids, np.int32)
        uh = np.ascontiguousarray(unique_hit, np.uint8)
        m = np.ascontiguousarray(miss_ids, np.int32)
        hs = np.empty(max(m.size, 1), np.int32)
        ld = np.empty(max(m.size, 1), np.uint8)
        check(lib().nvmoe_host_tier_resolve(self.h, u.ctypes.data, uh.ctypes.data, u.size,
                                            m.ctypes.data, m.size, hs.ctypes.data, ld.ctypes.data),
              "nvmoe_host_tier_resolve")
        return hs[:m.size], ld[:m.size]

    def stats(self) -> tuple[int, int]:
        """(host hits, host misses) over every resolve call (nvmoe_host_tier_stats)."""
        hh, hm = C.c_int64(0), C.c_int64(0)
        check(lib().nvmoe_host_tier_stats(self.h, C.byref(hh), C.byref(hm)),
              "nvmoe_host_tier_stats")
        return hh.value, hm.value

    def tables(self):
        a = np.empty(self.n_expert, np.int32)
        b = np.empty(self.host_slots, np.int32)
        check(lib().nvmoe_host_tier_tables(self.h, a.ctypes.data, b.ctypes.data),
              "nvmoe_host_tier_tables")
        return a, b


def _empty_like_slots(w: ExpertWeights, n: int, pin: bool) -> ExpertWeights:
    def mat(m: QuantMatrix) -> QuantMatrix:
        def z(t):
            if t is None:
                return None
            out = torch.zeros((n,) + tuple(t.shape[1:]), dtype=t.dtype)
            return out.pin_memory() if pin else out
        return QuantMatrix(m.quant, m.rows, m.cols, z(m.data), z(m.scale), z(m.glob))
    return ExpertWeights(w.quant, w.hidden, w.inter, mat(w.gate_up), mat(w.down))


def _bank_tensors(w: ExpertWeights):
    out = []
    for m in (w.gate_up, w.down):
        for t in (m.data, m.scale, m.glob):
            if t is not None:
                out.append(t)
    return out


class BoundedTierStack:
    """cfg.n_layers dependent decode layers (router gate, top-k, remap, host tier, side-stream
    refill, expert FFN) over GPU pools of cfg.cache_size slots and per-layer pinned host tiers of
    host_slots experts in front of a backing store holding every expert (shared by the layers,
    like the synthetic weights).  Eager: the host reads each layer step's miss list."""

    def __init__(self, cfg, host_slots: int, backing: ExpertWeights | None = None,
                 device="cuda", seed: int = 0, protected_ratio: float = 0.8, loader=None):
        """loader: where host-tier misses are read from instead of `backing` (an object with
        load_into(layer, expert, host_banks, host_slot), e.g. loaders.FtwModel or
        loaders.InterleavedSidecar); `backing` still gives the pools' shapes."""
        from .engine import MoEStack
        from .formats import random_experts
        self.cfg, self.host_slots = cfg, host_slots
        self.loader = loader
        self.device = d = torch.device(device)
        self.backing = backing if backing is not None else random_experts(
            cfg.quant, cfg.n_experts, cfg.hidden, cfg.inter, seed=seed)
        # the engine's pools, tables, shared experts and router gates; its own host tier (all
        # experts) is not used by this stack
        self.core = MoEStack(dataclasses.replace(cfg), device=d, seed=seed + 1,
                             host_tier=_empty_like_slots(self.backing, 1, pin=False))
        L = cfg.n_layers
        self.host = [_empty_like_slots(self.backing, host_slots, pin=True) for _ in range(L)]
        self.tiers = [HostTier(cfg.n_experts, host_slots, protected_ratio) for _ in range(L)]
        self.banks = [ops.refill_banks(self.core.pools[l], self.host[l]) for l in range(L)]
        self.copy_stream = torch.cuda.Stream(d)
        self.done = torch.cuda.Event()
        n_cap = cfg.n_experts
        self.misses = ops.MissListGPU(n_cap, d)
        self.stage = torch.empty(4 + 5 * n_cap, dtype=torch.int32).pin_memory()
        self.stats = {"gpu_misses": 0, "host_hits": 0, "host_loads": 0, "refill_bytes": 0,
                      "steps": 0}
        self._buf: dict[int, dict] = {}

    def init_router(self, logit_bias=None, seed: int = 0, eps: float = 1e-6) -> None:
        self.core.init_router(logit_bias=logit_bias, seed=seed, eps=eps)

    def buffers(self, n: int) -> dict:
        if n not in self._buf:
            c, d = self.cfg, self.device
            self._buf[n] = {
                "h": torch.empty((c.n_layers, n, c.hidden), dtype=torch.bfloat16, device=d),
                "xn": torch.empty((c.n_layers, n, c.hidden), dtype=torch.bfloat16, device=d),
                "logits": torch.empty((c.n_layers, n, c.n_experts), dtype=torch.float32,
                                      device=d),
                "y": torch.empty((c.n_layers, n, c.hidden), dtype=torch.bfloat16, device=d),
                "ids": torch.empty((c.n_layers, n, c.top_k), dtype=torch.int32, device=d),
                "w": torch.empty((c.n_layers, n, c.top_k), dtype=torch.float32, device=d),
                "slots": torch.empty((c.n_layers, n, c.top_k), dtype=torch.int32, device=d),
                "ws": ops.FfnWorkspace(d)}
        return self._buf[n]

    def _load(self, l: int, expert: int, host_slot: int) -> None:
        """Backing store -> pinned host slot (the stand-in for the NVMe read): a read from the
        model's files when the stack has a loader, else a copy from the in-memory store."""
        if self.loader is not None:
            self.loader.load_into(l, expert, _bank_tensors(self.host[l]), host_slot)
            return
        for dst, src in zip(_bank_tensors(self.host[l]), _bank_tensors(self.backing)):
            dst[host_slot].copy_(src[expert])

    def layer_step(self, l: int, x: torch.Tensor, resid: torch.Tensor | None, b: dict,
                   trace: list | None = None) -> None:
        c = self.cfg
        core = self.core
        ops.router_gate(resid if resid is not None else x, core.gate_w[l],
                        delta=b["y"][l - 1] if (l >= 1 and resid is not None) else None,
                        norm_weight=core.norm_w[l], eps=core.eps,
                        logit_bias=None if core.logit_bias is None else core.logit_bias[l],
                        resid_out=b["h"][l], x_out=b["xn"][l], logits=b["logits"][l])
        ops.router_topk(b["logits"][l], c.top_k, out_ids=b["ids"][l], out_weights=b["w"][l])
        ops.remap(core.tables[l], b["ids"][l], is_decode=True, out=b["slots"][l],
                  misses=self.misses)
        # the miss list to the host (eval_cb's per-layer read-back)
        m = self.misses
        cap = m.capacity
        st = self.stage
        st[:4].copy_(m.counts, non_blocking=True)
        st[4:4 + cap].copy_(m.unique_ids, non_blocking=True)
        st[4 + cap:4 + 2 * cap].copy_(m.unique_hit.to(torch.int32), non_blocking=True)
        st[4 + 2 * cap:4 + 3 * cap].copy_(m.miss_ids, non_blocking=True)
        st[4 + 3 * cap:4 + 4 * cap].copy_(m.miss_slots, non_blocking=True)
        torch.cuda.current_stream(self.device).synchronize()
        cnt = st[:4].numpy()
        if cnt[2] != 0:
            raise _lib.NvmoeError(int(cnt[2]), "nvmoe_remap")
        nu, nm = int(cnt[0]), int(cnt[1])
        s = st.numpy()
        uid, uhit = s[4:4 + nu], s[4 + cap:4 + cap + nu].astype(np.uint8)
        mid, msl = s[4 + 2 * cap:4 + 2 * cap + nm], s[4 + 3 * cap:4 + 3 * cap + nm]
        hs, ld = self.tiers[l].resolve(uid, uhit, mid)
        for j in range(nm):
            if ld[j]:
                self._load(l, int(mid[j]), int(hs[j]))
        if trace is not None:
            trace.append({"miss_ids": mid.copy(), "miss_slots": msl.copy(), "host_slots": hs.copy(),
                          "loads": ld.copy()})
        if nm:
            ops.refill_async(self.banks[l], msl, hs, c.cache_size, self.host_slots,
                             self.copy_stream, torch.cuda.current_stream(self.device), self.done)
        self.stats["gpu_misses"] += nm
        self.stats["host_loads"] += int(ld.sum())
        self.stats["host_hits"] += nm - int(ld.sum())
        self.stats["refill_bytes"] += nm * core.bytes_per_expert
        ops.moe_ffn(core.pools[l], b["xn"][l], b["slots"][l], b["w"][l], shared=core.shared[l],
                    out=b["y"][l], workspace=b["ws"])

    def forward(self, x: torch.Tensor, out: torch.Tensor, trace: list | None = None):
        """Dependent layers on tokens x [n, H]; out = the residual after the last layer."""
        n = x.shape[0]
        b = self.buffers(n)
        for l in range(self.cfg.n_layers):
            resid = None if l == 0 else (x if l == 1 else b["h"][l - 1])
            self.layer_step(l, x, resid, b, trace)
        L = self.cfg.n_layers
        ops.residual_add(x if L == 1 else b["h"][L - 1], b["y"][L - 1], out)
        self.stats["steps"] += 1
        return out
