"""Expert parallelism on 2 GPUs (NCCL): each rank owns half of the experts in its own slot pool
and the routed pairs travel by all-to-all (nvmoe_b200.ep); every rank's output matches the
single-GPU FFN over the full pool on the same tokens, within the FFN tolerance.  Skipped with
fewer than 2 GPUs."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
E, K, H, I = 16, 4, 2048, 512


def _worker(rank, world, port, q):
    import datetime
    from nvmoe_b200 import ops
    from nvmoe_b200.engine import _slot_view
    from nvmoe_b200.ep import ep_layer, nvmoe_local_ffn
    from nvmoe_b200.formats import random_experts
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    try:
        full = random_experts("nvfp4", E, H, I, seed=91).to(dev)
        shared = random_experts("nvfp4", 1, H, I, seed=92).to(dev)
        per = E // world
        local_pool = _slot_view(full, rank * per, per)
        table = ops.SlotTableGPU(per, per, dev)
        table.slot_of_real.copy_(torch.arange(per, dtype=torch.int32))   # all local experts resident
        table.real_in_slot.copy_(torch.arange(per, dtype=torch.int32))
        local = nvmoe_local_ffn(local_pool, table)
        one = torch.zeros((1,), dtype=torch.int32, device=dev)
        errs = []
        for step in range(3):
            rng = np.random.default_rng(1000 * rank + step)
            B = 3 + rank
            ids = torch.from_numpy(np.stack([rng.choice(E, size=K, replace=False)
                                             for _ in range(B)]).astype(np.int32)).to(dev)
            w = torch.from_numpy(rng.random((B, K)).astype(np.float32)).to(dev)
            x = torch.from_numpy(rng.standard_normal((B, H)).astype(np.float32)).to(
                torch.bfloat16).to(dev)
            shared_ffn = lambda t: ops.moe_ffn(shared, t, one.expand(t.shape[0], 1).contiguous(),
                                               torch.ones((t.shape[0], 1), device=dev))
            y = ep_layer(x, ids, w, E, local, shared_ffn=shared_ffn)
            ref = ops.moe_ffn(full, x, ids, w, shared=shared)
            torch.cuda.synchronize()
            yv, rv = y.float().cpu().numpy(), ref.float().cpu().numpy()
            errs.append(float(np.abs(yv - rv).max() / np.abs(rv).max()))
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


def test_ep_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for r in range(2):
        assert max(res[r]) <= 1e-2, res
