"""Expert-parallel dispatch / combine (nvmoe_b200.ep.ep_layer) on 2 and 4 gloo ranks (CPU): every
rank's output equals the single-process MoE over all experts, with uneven pair counts, a rank
that receives no pairs, and the shared expert.  The local expert step is a torch stand-in
(y = w * x @ W_e) so only the host-side partitioning and exchange are under test."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nvmoe_b200.ep import ep_layer, expert_owner

E, K, H = 8, 3, 16


def _weights():
    g = torch.Generator().manual_seed(5)
    return torch.randn((E, H, H), generator=g), torch.randn((H, H), generator=g)


def _tokens(rank, case):
    g = torch.Generator().manual_seed(100 + rank + 10 * case)
    B = 5 + 2 * rank
    x = torch.randn((B, H), generator=g)
    if case == 1:  # every pair goes to rank 0's experts: rank 1 receives nothing
        ids = torch.stack([torch.randperm(E // 2, generator=g)[:K] for _ in range(B)])
    else:
        ids = torch.stack([torch.randperm(E, generator=g)[:K] for _ in range(B)])
    w = torch.rand((B, K), generator=g)
    return x, ids.to(torch.int32), w


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        W, Ws = _weights()
        per = E // world
        out = []
        for case in (0, 1):
            x, ids, w = _tokens(rank, case)

            def local(xp, eid, wp):
                assert int(eid.min()) >= 0 and int(eid.max()) < per
                return wp[:, None] * torch.bmm(xp[:, None, :], W[rank * per + eid.long()])[:, 0]

            y = ep_layer(x, ids, w, E, local, shared_ffn=lambda t: t @ Ws)
            ref = Ws.new_zeros(x.shape) + x @ Ws
            for j in range(K):
                ref += w[:, j:j + 1] * torch.bmm(x[:, None, :], W[ids[:, j].long()])[:, 0]
            out.append(float((y - ref).abs().max()))
        q.put((rank, out))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("world", [2, 4])
def test_ep_layer_ranks_match_single_process(world):
    """2 and 4 ranks (4: two ranks receive nothing in the skewed case)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for r in range(world):
        assert max(res[r]) < 1e-4, res


def test_expert_owner_contiguous_shards():
    ids = torch.arange(E)
    assert expert_owner(ids, E, 4).tolist() == [0, 0, 1, 1, 2, 2, 3, 3]


def test_uneven_shards_are_rejected():
    """n_expert must be a positive multiple of the world size: a shard of E // P experts with a
    remainder would route the tail experts to rank P, which does not exist."""
    with pytest.raises(ValueError):
        expert_owner(torch.arange(10), 10, 4)
    with pytest.raises(ValueError):
        expert_owner(torch.arange(3), 3, 4)


def _reject_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x = torch.zeros((2, H))
        ids = torch.zeros((2, K), dtype=torch.int32)
        try:
            ep_layer(x, ids, torch.ones((2, K)), 7, lambda a, b, c: a)
            q.put((rank, "no error"))
        except ValueError:
            q.put((rank, "rejected"))
    finally:
        dist.destroy_process_group()


def test_ep_layer_rejects_uneven_shards_on_gloo_ranks():
    """Both ranks refuse 7 experts over 2 ranks before any collective runs."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_reject_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
    assert res == {0: "rejected", 1: "rejected"}
