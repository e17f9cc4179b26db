"""Drop-in for the Python engine's offload-cache surface on the routed-expert path.

Mirrors `NvmeOffloadMoeCache` (nvme-moe-bench/nvme_offload_cache.py:441) as the engine's decode
and narrow-prefill patches drive it (`patched_decode_routed`, :2142-2184; the prefill narrow
patch, :1957-2013):

  ensure_experts(layer_id, expert_ids)  expert ids -> global slot ids, in place (:1366)
  copy_missing()                        copies the last ensure's misses into their slots (:1684)
  bank_views(n=None)                    the slot pool's banks, FTW order (:954)
  alphas_for_slots(layer_id)            None, as in the reference (:959)
  slot_for_id                           [L, E] int32 slot of each expert, -1 = not resident
  id_of_slot                            [S] int32 global id (layer * E + e) in each slot
  reset(), is_cpu_layer(layer_id), cache_size, num_layers, num_experts, prefill_overlap,
  decode_target

and `expert_gemm(cache, hidden, topk_weights, slot_ids, views, n, alphas, is_prefill)`, the
engine's `_expert_gemm` call (:1989-1998, :2165-2174), with the two call sequences of the
engine's patches: `decode_routed` (:2142-2184) and the narrowed `prefill_routed` (:1957-2013);
`materialize_layer` (:1626) is the non-narrowed prefill's full-layer sweep.

Slots are global across layers and `cache_size >= num_experts`, as the reference requires
(:456-457).  The slot tables are the remap kernel's device arrays with `id_base = layer * E`.
The victim rule is eval_cb's (scripts/moe_cache_probe.cpp:627-753): the Python engine's own
`lru_ensure` order is not pinned by any reference test.

The host tier holds every expert of every layer in pinned memory, rows in global-id order.  The
reference's bounded host tier with NVMe backing is outside this path, and misses are copied
from the host tier by the SM gather kernel.

Nothing here synchronises the host with the device: remap errors (slot-pool overflow, a bad id)
stay in the device status until `check()` reads them.
"""
from __future__ import annotations

import numpy as np
import torch

from . import ops
from .formats import ExpertWeights, QuantMatrix


class SlotCache:
    def __init__(self, host_tier: ExpertWeights, num_layers: int, num_experts: int,
                 cache_size: int, device="cuda"):
        if cache_size < num_experts:  # the reference's own check (nvme_offload_cache.py:456)
            raise ValueError(f"cache_size {cache_size} < num_experts {num_experts}")
        if host_tier.n_slots != num_layers * num_experts:
            raise ValueError(f"host tier holds {host_tier.n_slots} experts, expected "
                             f"num_layers * num_experts = {num_layers * num_experts}")
        self.num_layers, self.num_experts, self.cache_size = num_layers, num_experts, cache_size
        self.device = torch.device(device)
        self.quant_format = host_tier.quant
        self.hidden, self.inter = host_tier.hidden, host_tier.inter
        self.prefill_overlap = False
        self.decode_target = "gpu"
        self.host = host_tier
        self.pool = _empty_pool(host_tier, cache_size, self.device)
        self.table = ops.SlotTableGPU(num_layers * num_experts, cache_size, self.device)
        self.misses = ops.MissListGPU(num_experts, self.device)
        self.host_slot_of_id = torch.arange(num_layers * num_experts, dtype=torch.int32,
                                            device=self.device)
        self.banks = ops.refill_banks(self.pool, host_tier)
        self._pending_layer: int | None = None

    # ---------------------------------------------------------------- tables
    @property
    def slot_for_id(self) -> torch.Tensor:
        return self.table.slot_of_real.view(self.num_layers, self.num_experts)

    @property
    def id_of_slot(self) -> torch.Tensor:
        return self.table.real_in_slot

    def is_cpu_layer(self, layer_id: int) -> bool:
        return False

    def reset(self) -> None:
        self.table.reset()
        self._pending_layer = None

    # ---------------------------------------------------------------- the hook
    def ensure_experts(self, layer_id: int, expert_ids: torch.Tensor) -> None:
        """Rewrites `expert_ids` (int32, any shape, last dim contiguous) to global slot ids in
        place and records the misses for copy_missing()."""
        if expert_ids.dtype != torch.int32:
            raise TypeError(f"expert_ids must be int32, got {expert_ids.dtype}")
        ids2 = expert_ids.view(1, -1) if expert_ids.dim() <= 1 else expert_ids.view(
            -1, expert_ids.shape[-1])
        n = ids2.numel()
        if self.misses.capacity < n:
            self.misses = ops.MissListGPU(n, self.device)
        ops.remap(self.table, ids2, is_decode=True, out=ids2, misses=self.misses,
                  id_base=layer_id * self.num_experts, n_expert=self.num_experts)
        self._pending_layer = layer_id

    def copy_missing(self) -> None:
        layer_id = self._pending_layer
        assert layer_id is not None, "copy_missing() without a preceding ensure_experts()"
        ops.refill_gather(self.banks, self.misses,
                          self.host_slot_of_id[layer_id * self.num_experts:], self.cache_size)
        self._pending_layer = None

    def bank_views(self, n: int | None = None) -> tuple[torch.Tensor, ...]:
        views = self.pool.banks()
        return views if n is None else tuple(v[:n] for v in views)

    def alphas_for_slots(self, layer_id: int):
        return None

    def materialize_layer(self, layer_id: int) -> None:
        """The non-narrowed prefill's full-layer sweep (nvme_offload_cache.py:1626-1682): every
        expert of layer_id is placed at its identity slot (expert e in slot e, the layout
        bank_views(num_experts) presents to the GEMM), evicting whatever those slots held, and
        its bytes are copied in from the host tier by the copy engine (nvmoe_refill_async)."""
        E = self.num_experts
        base = layer_id * E
        old = self.table.real_in_slot[:E].clone()
        held = old >= 0
        self.table.slot_of_real[old[held].long()] = -1
        ident = torch.arange(E, dtype=torch.int32, device=self.device)
        self.table.slot_of_real[base:base + E] = ident
        self.table.real_in_slot[:E] = ident + base
        step = int(self.table.step.item()) + 1
        self.table.step.fill_(step)
        self.table.last_used[:E] = step
        cs = torch.cuda.Stream(self.device)
        ev = torch.cuda.Event()
        ops.refill_async(self.banks, np.arange(E, dtype=np.int32),
                         np.arange(base, base + E, dtype=np.int32), self.cache_size,
                         self.host.n_slots, cs, torch.cuda.current_stream(self.device), ev)
        self._pending_layer = None

    def check(self) -> None:
        """Raises if the last remap reported an error (reads the device status: synchronises)."""
        st = int(self.misses.counts[2].item())
        if st != 0:
            raise RuntimeError(f"nvmoe remap failed with status {st}")


def expert_gemm(cache: SlotCache, hidden: torch.Tensor, topk_weights: torch.Tensor,
                slot_ids: torch.Tensor, views, n, alphas, is_prefill: bool) -> torch.Tensor:
    """The engine's `_expert_gemm` (nvme_offload_cache.py:1989-1998, 2165-2174):
    y[t] = sum_j w[t,j] * down_s(silu(gate_s x) * up_s x) over the banks in `views` (their first
    n slots when n is given), s = slot_ids[t, j] (routed experts only; the shared expert is the
    caller's, as in the reference).  is_prefill selects the token-sorted tcgen05 grouped GEMM
    (nvmoe_moe_ffn_prefill), else the decode kernel (nvmoe_moe_ffn).  bf16 in / out, fp32
    accumulation."""
    if alphas is not None:
        raise NotImplementedError("per-slot alphas: the FTW banks carry their global scales")
    if n is not None:
        views = tuple(v[:n] for v in views)
    pool = pool_from_views(views, cache.quant_format, cache.hidden, cache.inter)
    ids = slot_ids.reshape(hidden.shape[0], -1)
    if ids.dtype != torch.int32:
        ids = ids.to(torch.int32)
    w = topk_weights.reshape(hidden.shape[0], -1).to(torch.float32).contiguous()
    if is_prefill and cache.quant_format == "nvfp4":
        return ops.moe_ffn_prefill(pool, hidden.contiguous(), ids.contiguous(), w)
    return ops.moe_ffn(pool, hidden.contiguous(), ids.contiguous(), w)


def decode_routed(cache: SlotCache, layer_id: int, hidden: torch.Tensor,
                  topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """The engine's patched decode step (nvme_offload_cache.py:2142-2184): ensure the routed
    experts (ids rewritten to slots in place), copy the misses in, then the expert GEMM."""
    cache.ensure_experts(layer_id, topk_ids)
    cache.copy_missing()
    return expert_gemm(cache, hidden, topk_weights, topk_ids, views=cache.bank_views(), n=None,
                       alphas=cache.alphas_for_slots(layer_id), is_prefill=False)


def prefill_routed(cache: SlotCache, layer_id: int, hidden: torch.Tensor,
                   topk_weights: torch.Tensor, topk_ids: torch.Tensor) -> torch.Tensor:
    """The narrowed prefill (nvme_offload_cache.py:1957-2013): the routed union of the whole
    prompt (topk_ids.unique(), ascending) is ensured in one call, its misses copied in, the
    full topk_ids mapped to slots with one slot_for_id gather, then the expert GEMM over the
    cache_size slots with is_prefill=True.  topk_ids is not modified."""
    union = topk_ids.reshape(-1).unique().to(torch.int32)
    cache.ensure_experts(layer_id, union)  # rewrites union in place; unused after
    cache.copy_missing()
    slot_ids = cache.slot_for_id.reshape(-1)[layer_id * cache.num_experts +
                                              topk_ids.long()].to(torch.int32)
    return expert_gemm(cache, hidden, topk_weights, slot_ids, views=cache.bank_views(),
                       n=cache.cache_size, alphas=cache.alphas_for_slots(layer_id),
                       is_prefill=True)


def pool_from_views(views, quant: str, hidden: int, inter: int) -> ExpertWeights:
    """ExpertWeights over the bank tensors of bank_views() (no copy): NVFP4 in FTW order
    (gate_up codes, scales, global, down codes, scales, global), the GGUF formats and bf16 as
    (gate_up, down) byte rows."""
    u8 = torch.uint8
    if quant == "nvfp4":
        gu, gus, gug, dn, dns, dng = views
        gate_up = QuantMatrix(quant, 2 * inter, hidden, gu, gus.view(u8), gug.reshape(-1))
        down = QuantMatrix(quant, hidden, inter, dn, dns.view(u8), dng.reshape(-1))
        return ExpertWeights(quant, hidden, inter, gate_up, down)
    if quant in ("q2_k", "iq2_xxs"):
        gu, dn = views
        return ExpertWeights(quant, hidden, inter, QuantMatrix(quant, 2 * inter, hidden, gu.view(u8)),
                             QuantMatrix(quant, hidden, inter, dn.view(u8)))
    if quant == "bf16":
        gu, dn = views
        n = gu.shape[0]
        return ExpertWeights(quant, hidden, inter,
                             QuantMatrix(quant, 2 * inter, hidden, gu.reshape(n, 2 * inter, -1).view(u8)),
                             QuantMatrix(quant, hidden, inter, dn.reshape(n, hidden, -1).view(u8)))
    raise NotImplementedError(f"{quant} pools in the FFN")


def _empty_pool(like: ExpertWeights, n_slots: int, device) -> ExpertWeights:
    def mat(m: QuantMatrix) -> QuantMatrix:
        return QuantMatrix(
            m.quant, m.rows, m.cols,
            torch.zeros((n_slots,) + tuple(m.data.shape[1:]), dtype=m.data.dtype, device=device),
            None if m.scale is None else torch.zeros((n_slots,) + tuple(m.scale.shape[1:]),
                                                     dtype=m.scale.dtype, device=device),
            None if m.glob is None else torch.zeros((n_slots,), dtype=m.glob.dtype,
                                                    device=device))
    return ExpertWeights(like.quant, like.hidden, like.inter, mat(like.gate_up), mat(like.down))
