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
