"""GPU parity of one fused decode layer step (nvmoe_decode_layer) against the oracle chain:
router top-k -> eval_cb remap (C oracle) -> refill from the host tier -> fp32 FFN."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.engine import MoEStack, StackConfig
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer

pytestmark = pytest.mark.gpu


def _dense(w, which, s):
    I = w.inter
    m = w.gate_up if which != "down" else w.down
    rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
    return R.dequant_nvfp4(m.data[s, rows].numpy(), m.scale[s, rows].numpy(), m.glob[s].item())


@pytest.mark.parametrize("n_tok,prewarm", [(1, False), (3, True), (4, False), (8, False)])
def test_decode_layer_matches_oracle_chain(cuda_device, n_tok, prewarm):
    cfg = StackConfig(n_layers=2, n_experts=64, top_k=4, hidden=2048, inter=512, cache_size=16)
    stack = MoEStack(cfg, device=cuda_device, seed=3)
    bias = layer_log_bias(2, 64, 1.1, seed=1)
    orc = [OracleLayer(64, 16), OracleLayer(64, 16)]
    if prewarm:
        rank = np.argsort(-bias, axis=1, kind="stable")
        stack.prewarm(rank)
        for l in range(2):
            for e in rank[l][:16]:
                orc[l].eval(np.array([e], np.int32), is_decode=False)
            # the prewarm installs slot s <- rank[s]; align the oracle's step / stamps
            sor, ris, lu, _ = orc[l].tables()
            orc[l].set_tables(sor, ris, np.zeros_like(lu), 0)
    host = stack.host
    # distinct global scales per expert (the synthetic banks share one), so a slot whose scale
    # were taken before the refill replaced its expert would show in y
    for m in (host.gate_up, host.down):
        m.glob.mul_(torch.from_numpy(2.0 ** (np.arange(64) % 5 - 2.0)).float())
    if prewarm:
        stack.prewarm(rank)
    cache = {}

    def hd(which, e):
        if (which, e) not in cache:
            cache[(which, e)] = _dense(host, which, e)
        return cache[(which, e)]

    rng = np.random.default_rng(n_tok)
    for step in range(12):
        for l in range(2):
            lg = router_logits(n_tok, bias[l], rng)
            x = torch.from_numpy(rng.standard_normal((n_tok, 2048)).astype(np.float32)).to(
                torch.bfloat16)
            y = stack.layer_step(l, x.to(cuda_device), torch.from_numpy(lg).to(cuda_device))
            plan = stack.plans(n_tok)[l]
            torch.cuda.synchronize()
            rids, rw = R.router_topk_softmax(lg, 4)
            ref = orc[l].eval(rids.reshape(-1), is_decode=True)
            if ref["status"] == -3:
                # more distinct experts than slots: the reference aborts (ubatch clamp,
                # moe_cache_probe.cpp:1668-1684); here the step reports the overflow, leaves the
                # tables untouched and outputs zeros
                assert int(plan.status.item()) == -3
                assert not y.float().abs().any()
                continue
            assert int(plan.status.item()) == 0
            assert ref["status"] == 0
            np.testing.assert_array_equal(plan.slot_ids.cpu().numpy().reshape(-1), ref["slots"])
            np.testing.assert_allclose(plan.weights.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
            h = plan.misses.to_host()
            np.testing.assert_array_equal(h["miss_ids"], ref["miss_ids"])
            # slot s now holds the host tier's expert (weights copied by the refill gather);
            # every routed expert's weights come from the host tier row of its id
            sw = stack.shared[l]
            sh = (_dense(sw.to("cpu"), "gate", 0), _dense(sw.to("cpu"), "up", 0),
                  _dense(sw.to("cpu"), "down", 0))
            yr = R.moe_ffn(x.view(torch.int16).numpy().view(np.uint16), rids, rw,
                           lambda e: hd("gate", e), lambda e: hd("up", e),
                           lambda e: hd("down", e), shared=sh)
            if not prewarm and step == 0:
                pass  # cold pool: every routed expert was a miss and came from the host tier
            yv = y.float().cpu().numpy()
            scale = float(np.abs(yr).max())
            assert np.abs(yv - yr).max() <= 1e-2 * scale


def test_decode_layer_graph_replay_equals_eager(cuda_device):
    cfg = StackConfig(n_layers=3, n_experts=64, top_k=4, hidden=2048, inter=512, cache_size=16)
    a = MoEStack(cfg, device=cuda_device, seed=5)
    b = MoEStack(cfg, device=cuda_device, seed=5, host_tier=a.host)
    rng = np.random.default_rng(9)
    lg = torch.from_numpy(rng.standard_normal((6, 3, 2, 64)).astype(np.float32)).to(cuda_device)
    xs = torch.randn((6, 2, 2048), device=cuda_device).to(torch.bfloat16)
    out_a = torch.empty((3, 2, 2048), dtype=torch.bfloat16, device=cuda_device)
    out_b = torch.empty_like(out_a)
    b.forward(xs[0], lg[0], out_b)  # warm-up allocations for capture
    torch.cuda.synchronize()
    b = MoEStack(cfg, device=cuda_device, seed=5, host_tier=a.host)
    b.plans(2)
    b.forward(xs[0], lg[0], out_b)
    for t in b.tables:
        t.reset()
    s = torch.cuda.Stream()
    graphs = []
    for r in range(6):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            b.forward(xs[r], lg[r], out_b)
        graphs.append(g)
    for r in range(6):
        a.forward(xs[r], lg[r], out_a)
        graphs[r].replay()
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b)
        for ta, tb in zip(a.tables, b.tables):
            assert torch.equal(ta.slot_of_real, tb.slot_of_real)


def test_decode_layers_back_to_back_equal_serialised(cuda_device):
    """Consecutive layer steps overlap (a layer's front kernel runs during the previous
    layer's FFN, writing the other workspace / miss-list set; misses are copied in by the FFN).
    Run back to back in a CUDA graph, the outputs and tables must equal those of the same
    steps run one layer at a time with the device idle in between."""
    cfg = StackConfig(n_layers=4, n_experts=64, top_k=4, hidden=2048, inter=512, cache_size=16)
    a = MoEStack(cfg, device=cuda_device, seed=7)
    b = MoEStack(cfg, device=cuda_device, seed=7, host_tier=a.host)
    n, steps = 8, 5
    rng = np.random.default_rng(4)
    bias = torch.from_numpy(layer_log_bias(4, 64, 1.1, seed=2)).to(cuda_device)
    lg = (torch.from_numpy(rng.standard_normal((steps, 4, n, 64)).astype(np.float32))
          .to(cuda_device) + bias[None, :, None, :])
    xs = torch.randn((steps, n, 2048), device=cuda_device).to(torch.bfloat16)
    out_a = torch.empty((4, n, 2048), dtype=torch.bfloat16, device=cuda_device)
    out_b = torch.empty_like(out_a)
    b.forward(xs[0], lg[0], out_b)  # allocations before capture
    torch.cuda.synchronize()
    b = MoEStack(cfg, device=cuda_device, seed=7, host_tier=a.host)
    b.plans(n)
    s = torch.cuda.Stream()
    graphs = []
    for r in range(steps):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            b.forward(xs[r], lg[r], out_b)
        graphs.append(g)
    for t in b.tables:
        t.reset()
    for r in range(steps):
        for l in range(4):
            a.layer_step(l, xs[r], lg[r, l], out_a[l])
            torch.cuda.synchronize()
        graphs[r].replay()
        torch.cuda.synchronize()
        assert torch.equal(out_a, out_b), f"step {r}"
        for ta, tb in zip(a.tables, b.tables):
            assert torch.equal(ta.slot_of_real, tb.slot_of_real)


@pytest.mark.parametrize("n_tok", [1, 32])
def test_decode_layer_cpu_plumbing_bf16(cuda_device, n_tok):
    """The CPU-plumbing layer (64 experts, top-4, H 1024, I 256, bf16 weights ~N(0, 0.02), a
    16-slot LRU pool, Zipf(1.1) routing) through the engine against the oracle chain.  The
    engine clamps the micro-batch as the llama.cpp engine does (moe_cache_probe.cpp:1668-1684):
    min(6, (16 - 4) // 4) = 3 tokens, so batch 32 runs as 11 micro-batches, each one remap call
    whose distinct experts fit the 16 slots; every step is checked (outputs of every token, and
    the slot tables after the step)."""
    from nvmoe_b200.engine import safe_ubatch
    ub = safe_ubatch(16, 4)
    assert ub == 3
    cfg = StackConfig(n_layers=1, n_experts=64, top_k=4, hidden=1024, inter=256, cache_size=16,
                      quant="bf16", shared_expert=False, ubatch=ub)
    stack = MoEStack(cfg, device=cuda_device, seed=11)
    orc = OracleLayer(64, 16)
    bias = layer_log_bias(1, 64, 1.1, seed=0)[0]
    host = stack.host

    def dense(which, e):
        m = host.gate_up if which != "down" else host.down
        rows = slice(0, 256) if which == "gate" else (slice(256, 512) if which == "up" else slice(None))
        return R.bf16_to_f32(m.data[e, rows].contiguous().view(torch.int16).numpy().view(np.uint16))

    rng = np.random.default_rng(n_tok)
    out = torch.empty((1, n_tok, 1024), dtype=torch.bfloat16, device=cuda_device)
    for step in range(6):
        lg = router_logits(n_tok, bias, rng)
        x = torch.from_numpy(rng.standard_normal((n_tok, 1024)).astype(np.float32)).to(torch.bfloat16)
        stack.forward(x.to(cuda_device), torch.from_numpy(lg).to(cuda_device)[None], out)
        torch.cuda.synchronize()
        rids, rw = R.router_topk_softmax(lg, 4)
        for a, b in stack.ubatches(n_tok):
            ref = orc.eval(rids[a:b].reshape(-1), is_decode=True)
            assert ref["status"] == 0  # the clamp keeps every micro-batch within the pool
        plan = stack.plans(stack.ubatches(n_tok)[-1][1] - stack.ubatches(n_tok)[-1][0])[0]
        assert int(plan.status.item()) == 0
        sor, ris, lu, st = orc.tables()
        np.testing.assert_array_equal(stack.tables[0].slot_of_real.cpu().numpy(), sor)
        np.testing.assert_array_equal(stack.tables[0].real_in_slot.cpu().numpy(), ris)
        np.testing.assert_array_equal(stack.tables[0].last_used.cpu().numpy().view(np.uint32), lu)
        yr = R.moe_ffn(x.view(torch.int16).numpy().view(np.uint16), rids, rw,
                       lambda e: dense("gate", e), lambda e: dense("up", e),
                       lambda e: dense("down", e))
        scale = float(np.abs(yr).max())
        assert np.abs(out[0].float().cpu().numpy() - yr).max() <= 1e-2 * scale
