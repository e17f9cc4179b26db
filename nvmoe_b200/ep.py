"""Expert parallelism: the routed experts of a layer sharded across ranks (one process per GPU),
tokens dispatched to the rank that owns each of their experts and the expert outputs combined
back on the token's home rank, over torch.distributed all-to-all (NCCL on GPUs, gloo on CPU).

Rank r owns experts [r * E / P, (r + 1) * E / P) with its own slot pool, slot tables and host
tier.  One layer step on every rank:

  1. route its own tokens (top-k over all E experts, replicated router weights);
  2. dispatch: every (token, k) pair goes to the owner of its expert, sorted by destination
     (stable, so a pair's position is a function of the routing alone), with its hidden row,
     its expert's local id and its router weight; the pair counts travel first;
  3. local: the received pairs are a batch of top-1 tokens for the rank's own pool
     (remap -> refill -> FFN with the router weight applied);
  4. combine: the outputs travel back the same way and the home rank sums each token's k
     outputs in the order j = 0..k-1, plus its shared expert (computed locally: every rank
     holds the shared expert).

The local expert FFN is a callable, so the dispatch / combine logic is the same with the CUDA
path (`nvmoe_local_ffn`) and with a reference FFN in tests.
"""
from __future__ import annotations

from typing import Callable

import torch
import torch.distributed as dist

LocalFfn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def shard_size(n_expert: int, world: int) -> int:
    """Experts per rank.  The shards are contiguous and equal, so world must divide n_expert
    (and not exceed it); anything else would send pairs to a rank that does not exist."""
    if world <= 0 or n_expert < world or n_expert % world != 0:
        raise ValueError(f"expert parallelism needs n_expert ({n_expert}) to be a positive "
                         f"multiple of the world size ({world})")
    return n_expert // world


def expert_owner(expert_ids: torch.Tensor, n_expert: int, world: int) -> torch.Tensor:
    """Rank that owns each expert (contiguous shards of n_expert / world experts)."""
    per = shard_size(n_expert, world)
    return torch.div(expert_ids, per, rounding_mode="floor")


def ep_layer(x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor, n_expert: int,
             local_ffn: LocalFfn, shared_ffn: Callable[[torch.Tensor], torch.Tensor] | None = None,
             group=None) -> torch.Tensor:
    """One expert-parallel MoE step for this rank's tokens x [B, H] with routed global expert
    ids [B, k] (int32) and router weights [B, k] (fp32); returns y [B, H] in x's dtype.

    local_ffn(x_pairs [n, H], local_expert_ids [n] int32, weights [n] fp32) -> [n, H] computes
    weight * expert(x) for the pairs this rank received; shared_ffn(x) -> [B, H] the shared
    expert (or None)."""
    world = dist.get_world_size(group)
    B, k = ids.shape
    H = x.shape[1]
    per = shard_size(n_expert, world)
    dev = x.device
    # 2. dispatch, pairs grouped by destination rank (stable: pair p = t * k + j in order)
    flat_ids = ids.reshape(-1).to(torch.int64)
    dest = torch.div(flat_ids, per, rounding_mode="floor")
    order = torch.sort(dest, stable=True).indices
    send_counts = torch.bincount(dest, minlength=world).to(torch.int64)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    sc, rc = send_counts.tolist(), recv_counts.tolist()
    tok = torch.div(order, k, rounding_mode="floor")
    send_x = x.index_select(0, tok).contiguous()
    send_eid = (flat_ids[order] - dest[order] * per).to(torch.int32).contiguous()
    send_w = weights.reshape(-1)[order].to(torch.float32).contiguous()
    n_recv = sum(rc)
    recv_x = torch.empty((n_recv, H), dtype=x.dtype, device=dev)
    recv_eid = torch.empty((n_recv,), dtype=torch.int32, device=dev)
    recv_w = torch.empty((n_recv,), dtype=torch.float32, device=dev)
    dist.all_to_all_single(recv_x, send_x, rc, sc, group=group)
    dist.all_to_all_single(recv_eid, send_eid, rc, sc, group=group)
    dist.all_to_all_single(recv_w, send_w, rc, sc, group=group)
    # 3. the received pairs through this rank's experts (weight applied)
    if n_recv:
        y_pairs = local_ffn(recv_x, recv_eid, recv_w)
    else:
        y_pairs = torch.empty((0, H), dtype=x.dtype, device=dev)
    # 4. back to the home ranks, then the sum over j in order (fp32)
    back = torch.empty((B * k, H), dtype=y_pairs.dtype, device=dev)
    dist.all_to_all_single(back, y_pairs.contiguous(), sc, rc, group=group)
    per_pair = torch.empty_like(back)
    per_pair[order] = back  # pair p's output at row p = t * k + j
    per_pair = per_pair.view(B, k, H).to(torch.float32)
    y = per_pair[:, 0].clone()
    for j in range(1, k):
        y += per_pair[:, j]
    if shared_ffn is not None:
        y += shared_ffn(x).to(torch.float32)
    return y.to(x.dtype)


def nvmoe_local_ffn(pool, table, misses=None, refill_banks=None, host_slot_of_id=None,
                    workspace=None) -> LocalFfn:
    """The CUDA local step for ep_layer: remap the received local expert ids to slots of this
    rank's pool (miss list on the device), copy misses from the rank's pinned host tier, then
    the decode FFN with top-1 per pair and the router weight applied."""
    from . import ops

    def run(xp: torch.Tensor, eid: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        ids = eid.view(-1, 1).contiguous()
        slots, ml = ops.remap(table, ids, is_decode=True, misses=misses)
        if refill_banks is not None:
            ops.refill_gather(refill_banks, ml, host_slot_of_id, table.cache_size)
        return ops.moe_ffn(pool, xp.contiguous(), slots, w.view(-1, 1).contiguous(),
                           workspace=workspace)
    return run


# ---------------------------------------------------------------- the CUDA expert-parallel stack
class EPMoEStack:
    """Rank `rank` of `world` in an expert-parallel stack of dependent MoE layers (the decode
    stack of MoEStack.forward_chain with its routed experts sharded by contiguous ranges).

    The rank keeps, per layer, a slot pool and slot tables over its per = E / world routed
    experts plus its copy of the shared expert (local id per), a pinned host tier of those
    per + 1 experts, and the replicated router gates.  One layer step for n_tok home tokens:
        nvmoe_router_gate (with its fused top-k) -> nvmoe_ep_dispatch
        -> exchange (all-to-all of world equal segments)
        -> nvmoe_decode_layer, pre-routed, over the world * n_tok received rows (top_k + 1
           entries each: remap, refill from the host tier, expert FFN)
        -> exchange back -> nvmoe_ep_combine
    Every buffer size is fixed by n_tok, so a step has no host synchronisation and can be
    captured in a CUDA graph (with the exchanges, when they are NCCL collectives).

    global_host: the model's routed experts (E, on the CPU); shared: its shared expert (1 slot,
    CPU); ranking: [L, E] global expert popularity (most popular first) for the prewarm."""

    def __init__(self, cfg, n_tok: int, rank: int, world: int, global_host, shared,
                 device="cuda", seed: int = 0, logit_bias=None, router_seed: int = 5,
                 eps: float = 1e-6):
        import dataclasses

        import numpy as np

        from . import ops
        from .engine import MoEStack, _pin
        from .formats import concat_experts, select_experts

        self.cfg, self.n_tok, self.rank, self.world = cfg, n_tok, rank, world
        self.per = per = shard_size(cfg.n_experts, world)
        self.device = d = torch.device(device)
        local = concat_experts(select_experts(global_host, range(rank * per, (rank + 1) * per)),
                               shared)
        lcfg = dataclasses.replace(cfg, n_experts=per + 1, cache_size=min(cfg.cache_size, per + 1),
                                   shared_expert=False)
        self.local = MoEStack(lcfg, device=d, seed=seed, host_tier=_pin(local))
        # replicated router gates (the same seed on every rank)
        self.local.cfg = dataclasses.replace(lcfg, n_experts=cfg.n_experts)
        self.local.init_router(logit_bias=logit_bias, seed=router_seed, eps=eps)
        self.local.cfg = lcfg
        L, H, E, k = cfg.n_layers, cfg.hidden, cfg.n_experts, cfg.top_k
        self.K1 = k + 1
        self.row = ops.ep_row_bytes(H, k)
        z = lambda *shape, dt: torch.empty(shape, dtype=dt, device=d)  # noqa: E731
        self.h = z(L, n_tok, H, dt=torch.bfloat16)
        self.xn = z(L, n_tok, H, dt=torch.bfloat16)
        self.logits = z(L, n_tok, E, dt=torch.float32)
        self.y = z(L, n_tok, H, dt=torch.bfloat16)
        self.ids = z(n_tok, k, dt=torch.int32)
        self.w = z(n_tok, k, dt=torch.float32)
        self.tickets = torch.zeros(((n_tok + 7) // 8,), dtype=torch.int32, device=d)
        self.send = torch.zeros((world, n_tok, self.row), dtype=torch.uint8, device=d)
        self.recv = torch.zeros((world, n_tok, self.row), dtype=torch.uint8, device=d)
        self.slot_of = z(n_tok, world, dt=torch.int32)
        self.ypair = z(world, n_tok, H, dt=torch.bfloat16)
        self.back = z(world, n_tok, H, dt=torch.bfloat16)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        rv = self.recv.view(world * n_tok, self.row)
        self.recv_x = rv[:, :2 * H].view(torch.bfloat16)
        self.recv_ids = rv[:, 2 * H:2 * H + 4 * self.K1].view(torch.int32)
        self.recv_w = rv[:, 2 * H + 4 * self.K1:2 * H + 8 * self.K1].view(torch.float32)
        st = self.local
        self.plans = [
            ops.DecodeLayerPlan(st.pools[l], st.tables[l], st.misses_sets[l % 2], world * n_tok,
                                self.K1, refill=st.banks[l], host_slot_of_id=st.host_slot_of_id,
                                workspace=st.ws_sets[l % 2], device=d)
            for l in range(L)]
        self.gates = []
        for l in range(L):
            self.gates.append(ops.router_gate_args(
                self.h[l - 1] if l >= 2 else self.xn[0], self.logits[l], st.gate_w[l],
                delta=self.y[l - 1] if l >= 1 else None,
                resid_out=self.h[l] if l >= 1 else None, norm_weight=st.norm_w[l], eps=eps,
                x_out=self.xn[l],
                logit_bias=None if st.logit_bias is None else st.logit_bias[l],
                route=(k, self.ids, self.w, self.tickets, "softmax", None, True, 1.0)))
        self._np = np

    # ------------------------------------------------------------ cache state
    def local_ranking(self, ranking):
        """Per-layer prewarm order of this rank's pool: the shared expert, then its routed
        experts in global popularity order."""
        np = self._np
        per, r = self.per, self.rank
        out = []
        for row in np.asarray(ranking):
            mine = [int(e) - r * per for e in row if r * per <= int(e) < (r + 1) * per]
            out.append([per] + mine)
        return np.asarray(out, np.int64)

    def prewarm(self, ranking) -> None:
        self.local.prewarm(self.local_ranking(ranking))

    # ------------------------------------------------------------ one layer, in phases
    def phase_dispatch(self, l: int, x: torch.Tensor) -> None:
        """Router gate (residual add, RMSNorm, gate GEMV, top-k) and the dispatch pack of layer
        l; x is the stack's input tokens (read by layers 0 and 1)."""
        from . import _lib, ops
        import ctypes as C
        ga = self.gates[l]
        if l <= 1:
            ga.resid, ga.resid_row_stride = x.data_ptr(), x.stride(0)
        _lib.check(_lib.lib().nvmoe_router_gate(C.byref(ga), ops._stream()), "nvmoe_router_gate")
        ops.ep_dispatch(self.xn[l], self.ids, self.w, self.cfg.n_experts, self.world, self.rank,
                        self.send, self.slot_of, with_shared=True, status=self.status)

    def phase_local(self, l: int) -> None:
        """The owner's step over the received rows: remap, refill, expert FFN."""
        self.plans[l].routed(self.recv_x, self.recv_ids, self.recv_w,
                             self.ypair.view(self.world * self.n_tok, -1))

    def phase_combine(self, l: int) -> None:
        from . import ops
        ops.ep_combine(self.back, self.slot_of, self.y[l])

    def finish(self, x: torch.Tensor, out: torch.Tensor) -> torch.Tensor:
        """out = h_{L-1} + y_{L-1} (the residual after the last layer)."""
        from . import _lib, ops
        import ctypes as C
        L = self.cfg.n_layers
        fin = ops.router_gate_args(x if L == 1 else self.h[L - 1], None, None,
                                   delta=self.y[L - 1], resid_out=out)
        _lib.check(_lib.lib().nvmoe_router_gate(C.byref(fin), ops._stream()), "nvmoe_router_gate")
        return out

    # ------------------------------------------------------------ the whole stack over NCCL
    def forward(self, x: torch.Tensor, out: torch.Tensor, group=None) -> torch.Tensor:
        """All layers for this rank's tokens x [n_tok, H]; out [n_tok, H] = the residual after
        the last layer.  Every rank calls it in step (two all-to-alls per layer)."""
        send = self.send.view(-1)
        recv = self.recv.view(-1)
        yp = self.ypair.view(-1)
        back = self.back.view(-1)
        for l in range(self.cfg.n_layers):
            self.phase_dispatch(l, x)
            dist.all_to_all_single(recv, send, group=group)
            self.phase_local(l)
            dist.all_to_all_single(back, yp, group=group)
            self.phase_combine(l)
        return self.finish(x, out)


def ep_forward_emulated(stacks: list, xs: list, outs: list) -> list:
    """The same layer steps for every rank of an expert-parallel group held in one process (one
    GPU), the all-to-all done by segment copies: rank r receives segment r of every rank's send
    buffer, in rank order.  Tests the kernels and the data layout without a second GPU."""
    W = len(stacks)
    for l in range(stacks[0].cfg.n_layers):
        for r in range(W):
            stacks[r].phase_dispatch(l, xs[r])
        for r in range(W):
            for s in range(W):
                stacks[r].recv[s].copy_(stacks[s].send[r])
        for r in range(W):
            stacks[r].phase_local(l)
        for r in range(W):
            for s in range(W):
                stacks[r].back[s].copy_(stacks[s].ypair[r])
        for r in range(W):
            stacks[r].phase_combine(l)
    return [stacks[r].finish(xs[r], outs[r]) for r in range(W)]


class EPPrefill:
    """Expert-parallel prefill of one MoE layer: rank `rank` of `world` holds its per = E / world
    routed experts and the shared expert resident in one pool (slot = local id), receives the
    tokens routed to them and runs them through nvmoe_moe_ffn_prefill (token-sorted tcgen05
    grouped GEMM), pre-routed with top_k + 1 entries per row (negative ids empty).  Tokens enter
    and leave by nvmoe_ep_dispatch / nvmoe_ep_combine around two all-to-alls, as in the decode
    stack.  With world == 1 the exchanges are the identity (the segments are the buffers)."""

    def __init__(self, n_expert: int, top_k: int, n_tok: int, rank: int, world: int, global_host,
                 shared, device="cuda"):
        from . import ops
        from .formats import concat_experts, select_experts
        self.E, self.k, self.n_tok, self.rank, self.world = n_expert, top_k, n_tok, rank, world
        self.per = per = shard_size(n_expert, world)
        d = self.device = torch.device(device)
        self.pool = concat_experts(select_experts(global_host, range(rank * per, (rank + 1) * per)),
                                   shared).to(d)
        H = self.H = global_host.hidden
        self.K1 = top_k + 1
        self.row = ops.ep_row_bytes(H, top_k)
        self.send = torch.zeros((world, n_tok, self.row), dtype=torch.uint8, device=d)
        self.recv = self.send if world == 1 else torch.zeros_like(self.send)
        self.slot_of = torch.empty((n_tok, world), dtype=torch.int32, device=d)
        self.ypair = torch.empty((world, n_tok, H), dtype=torch.bfloat16, device=d)
        self.back = self.ypair if world == 1 else torch.empty_like(self.ypair)
        self.status = torch.zeros(1, dtype=torch.int32, device=d)
        rv = self.recv.view(world * n_tok, self.row)
        self.recv_x = rv[:, :2 * H].view(torch.bfloat16)
        self.recv_ids = rv[:, 2 * H:2 * H + 4 * self.K1].view(torch.int32)
        self.recv_w = rv[:, 2 * H + 4 * self.K1:2 * H + 8 * self.K1].view(torch.float32)
        self.ws = ops.FfnWorkspace(d)

    def forward(self, x: torch.Tensor, ids: torch.Tensor, weights: torch.Tensor,
                out: torch.Tensor, group=None) -> torch.Tensor:
        """This rank's n_tok tokens x [n_tok, H] with routed global ids / weights [n_tok, k]
        -> out [n_tok, H] (routed experts + shared expert).  Every rank calls it in step."""
        from . import ops
        ops.ep_dispatch(x, ids, weights, self.E, self.world, self.rank, self.send, self.slot_of,
                        with_shared=True, status=self.status)
        if self.world > 1:
            dist.all_to_all_single(self.recv.view(-1), self.send.view(-1), group=group)
        ops.moe_ffn_prefill(self.pool, self.recv_x, self.recv_ids, self.recv_w,
                            out=self.ypair.view(self.world * self.n_tok, self.H), workspace=self.ws,
                            status=self.status)
        if self.world > 1:
            dist.all_to_all_single(self.back.view(-1), self.ypair.view(-1), group=group)
        return ops.ep_combine(self.back, self.slot_of, out)
