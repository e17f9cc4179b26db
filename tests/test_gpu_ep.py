"""Expert parallelism on 2 GPUs over NCCL (nvmoe_b200.ep.EPMoEStack.forward): each rank owns
half of the 512 experts of the Qwen3.8 decode layer (plus its copy of the shared expert) in its
own 128-slot pools; tokens travel by two all-to-alls per layer.  Every rank's output is checked
against the oracle chain of the unsharded model (MoE output of each layer within
max |y - ref| <= 1e-2 max |ref|), and equals, bit for bit, the same ranks run in one process
with the exchange done by copies (ep_forward_emulated).  A second test replays the whole
two-rank stack, NCCL calls included, from a CUDA graph and compares it with the eager run.
Skipped with fewer than 2 GPUs.  NVLS is off (NCCL_NVLS_ENABLE=0)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
E, K, H, I, L, B = 512, 10, 2048, 512, 2, 8


def _model():
    from nvmoe_b200.engine import StackConfig
    from nvmoe_b200.formats import random_experts
    from nvmoe_b200.synth import layer_log_bias
    cfg = StackConfig(n_layers=L, n_experts=E, top_k=K, hidden=H, inter=I, cache_size=128)
    host = random_experts("nvfp4", E, H, I, seed=41)
    shared = random_experts("nvfp4", 1, H, I, seed=42)
    bias = layer_log_bias(L, E, 1.1, seed=3)
    return cfg, host, shared, bias


def _tokens(rank, step):
    rng = np.random.default_rng(100 * rank + step)
    return torch.from_numpy(rng.standard_normal((B, H)).astype(np.float32)).to(torch.bfloat16)


def _worker(rank, world, port, q, graph):
    import datetime
    from nvmoe_b200.ep import EPMoEStack
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    dev = torch.device("cuda", rank)
    dist.init_process_group("nccl", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60), device_id=dev)
    gr = None
    try:
        cfg, host, shared, bias = _model()
        st = EPMoEStack(cfg, B, rank, world, host, shared, device=dev, seed=7 + rank,
                        logit_bias=bias)
        st.prewarm(np.argsort(-bias, axis=1, kind="stable"))
        out = torch.empty((B, H), dtype=torch.bfloat16, device=dev)
        res = []
        if not graph:
            for step in range(2):
                x = _tokens(rank, step).to(dev)
                st.forward(x, out)
                torch.cuda.synchronize()
                res.append((out.cpu(), [st.y[l].cpu() for l in range(L)],
                            [st.xn[l].cpu() for l in range(L)], [st.logits[l].cpu() for l in range(L)],
                            [st.h[l].cpu() for l in range(L)]))
        else:
            x = _tokens(rank, 0).to(dev)
            st.forward(x, out)  # eager: allocations, then the same starting state again
            torch.cuda.synchronize()
            st.prewarm(np.argsort(-bias, axis=1, kind="stable"))
            eager = out.clone()
            st.prewarm(np.argsort(-bias, axis=1, kind="stable"))
            s = torch.cuda.Stream(dev)
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=s):
                st.forward(x, out)
            torch.cuda.synchronize()
            out.zero_()
            gr.replay()
            torch.cuda.synchronize()
            res.append((eager.cpu(), out.cpu()))
        q.put((rank, res))
    finally:
        gr = None
        dist.destroy_process_group()


def _run(graph):
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q, graph)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=600) for _ in procs)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


def test_ep_two_gpus_nccl_matches_oracle_and_emulation():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    from nvmoe_b200.ep import EPMoEStack, ep_forward_emulated
    from oracle import ref_numpy as R
    from tests.helpers import DenseExperts, bf16_bits, within
    res = _run(graph=False)
    cfg, host, shared, bias = _model()
    dense, sh = DenseExperts(host), DenseExperts(shared).shared(0)
    for r in range(2):
        for step, (out, ys, xns, lgs, hs) in enumerate(res[r]):
            for l in range(L):
                rids, rw = R.router_topk_softmax(lgs[l].numpy(), K)
                yr = R.moe_ffn(bf16_bits(xns[l]), rids, rw, *dense.callables(), shared=sh)
                assert within(ys[l], yr) <= 1e-2, (r, step, l)
    # the same two ranks in one process on GPU 0, exchanged by copies: identical bits
    dev = torch.device("cuda", 0)
    stacks = [EPMoEStack(cfg, B, r, 2, host, shared, device=dev, seed=7 + r, logit_bias=bias)
              for r in range(2)]
    for st in stacks:
        st.prewarm(np.argsort(-bias, axis=1, kind="stable"))
    outs = [torch.empty((B, H), dtype=torch.bfloat16, device=dev) for _ in range(2)]
    for step in range(2):
        ep_forward_emulated(stacks, [_tokens(r, step).to(dev) for r in range(2)], outs)
        torch.cuda.synchronize()
        for r in range(2):
            assert torch.equal(outs[r].cpu(), res[r][step][0]), (r, step)


def test_ep_two_gpus_graph_replay_equals_eager():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    res = _run(graph=True)
    for r in range(2):
        eager, replay = res[r][0]
        assert torch.equal(eager, replay), r
