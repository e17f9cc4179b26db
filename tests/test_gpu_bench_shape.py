"""Oracle parity of the timed paths at the benchmark's own shapes.

Decode: the Qwen3.8-shaped NVFP4 stack the decode benchmark times (512 experts, softmax top-10
with Zipf(1.1) skew, H 2048, I 512, a shared expert, 128 slots per layer) at batch 1, 8 and 64:
4 layers back to back in CUDA graphs with the alternating workspace / miss-list sets
(early_outputs), a pool prewarmed with ranks 32..159 of each layer's popularity so the hottest
experts miss and are copied in by the FFN from the pinned host tier, distinct global scales per
expert.  Every layer step is checked against the oracle chain: router ids and weights, the slot
ids, the slot tables after the step (which fix every miss and eviction), the miss list of the
last two layers (the two sets' final contents), and the FFN output.

Prefill: one layer of 4096 tokens over all 512 experts (top-10 Zipf routing, shared expert)
through nvmoe_moe_ffn_prefill, both tcgen05 kernels, against the fp32 oracle.

Tolerances: router weights rtol 2e-6; slot ids, tables and miss lists bit-exact; FFN outputs
max |y - ref| <= 1e-2 * max |ref| (fp32-accumulated oracle, bf16 output).
"""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.engine import MoEStack, StackConfig
from nvmoe_b200.formats import random_experts
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer
from tests.helpers import DenseExperts, bf16_bits, within

pytestmark = pytest.mark.gpu

E, K, H, I, S = 512, 10, 2048, 512, 128
FFN_TOL = 1e-2


def _distinct_globals(w, n):
    f = torch.from_numpy((2.0 ** (np.arange(n) % 5 - 2.0)).astype(np.float32))
    for m in (w.gate_up, w.down):
        m.glob.mul_(f.to(m.glob.device))


@pytest.mark.parametrize("batch,rounds", [(1, 6), (8, 4), (64, 3)])
def test_decode_stack_matches_oracle_at_bench_shape(cuda_device, batch, rounds):
    L = 4
    stack = MoEStack(StackConfig(n_layers=L), device=cuda_device, seed=21)
    _distinct_globals(stack.host, E)
    bias = layer_log_bias(L, E, 1.1, seed=0)
    rank = np.argsort(-bias, axis=1, kind="stable")
    warm = rank[:, 32:32 + S]  # the 32 hottest experts of each layer start out missing

    rng = np.random.default_rng(100 + batch)
    lg_h = np.stack([np.stack([router_logits(batch, bias[l], rng) for l in range(L)])
                     for _ in range(rounds)])  # [R, L, B, E]
    x_h = torch.from_numpy(rng.standard_normal((rounds, batch, H)).astype(np.float32)).to(
        torch.bfloat16)
    lg = torch.from_numpy(lg_h).to(cuda_device)
    xs = x_h.to(cuda_device)
    out = torch.empty((L, batch, H), dtype=torch.bfloat16, device=cuda_device)

    # eager pass (kernel attributes, allocations), then the starting state and the graphs
    stack.forward(xs[0], lg[0], out)
    torch.cuda.synchronize()
    stack.prewarm(warm)
    graphs, cap = [], torch.cuda.Stream(cuda_device)
    for r in range(rounds):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            stack.forward(xs[r], lg[r], out)
        graphs.append(g)
    torch.cuda.synchronize()

    orc = []
    for l in range(L):
        o = OracleLayer(E, S)
        sor = np.full(E, -1, np.int32)
        sor[warm[l]] = np.arange(S, dtype=np.int32)
        o.set_tables(sor, warm[l].astype(np.int32), np.zeros(S, np.uint32), 0)
        orc.append(o)
    dense = DenseExperts(stack.host)
    shared = [DenseExperts(stack.shared_all).shared(l) for l in range(L)]
    plans = stack.plans(batch)
    total_miss = 0
    for r in range(rounds):
        graphs[r].replay()
        torch.cuda.synchronize()
        for l in range(L):
            plan = plans[l]
            rids, rw = R.router_topk_softmax(lg_h[r, l], K)
            ref = orc[l].eval(rids.reshape(-1), is_decode=True)
            assert ref["status"] == 0
            assert int(plan.status.item()) == 0, (r, l)
            np.testing.assert_array_equal(plan.slot_ids.cpu().numpy().reshape(-1), ref["slots"])
            np.testing.assert_allclose(plan.weights.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
            sor, ris, lu, step = orc[l].tables()
            t = stack.tables[l]
            np.testing.assert_array_equal(t.slot_of_real.cpu().numpy(), sor)
            np.testing.assert_array_equal(t.real_in_slot.cpu().numpy(), ris)
            np.testing.assert_array_equal(t.last_used.cpu().numpy().view(np.uint32), lu)
            assert int(t.step.item()) == step
            total_miss += len(ref["miss_ids"])
            if l >= L - 2:  # set l % 2 still holds this layer's miss list
                h = stack.misses_sets[l % 2].to_host()
                np.testing.assert_array_equal(h["miss_ids"], ref["miss_ids"])
                np.testing.assert_array_equal(h["miss_slots"], ref["miss_slots"])
                np.testing.assert_array_equal(h["evicted"], ref["evicted"])
                np.testing.assert_array_equal(h["unique_ids"], ref["unique_ids"])
            # every routed expert's weights are the host tier's row of its id
            yr = R.moe_ffn(bf16_bits(x_h[r]), rids, rw, *dense.callables(), shared=shared[l])
            err = within(out[l], yr)
            assert err <= FFN_TOL, (r, l, err)
    assert total_miss > 0  # the in-FFN refill path ran


@pytest.fixture(scope="module")
def prefill_case(cuda_device):
    T = 4096
    pool = random_experts("nvfp4", E, H, I, seed=11)
    _distinct_globals(pool, E)
    shared = random_experts("nvfp4", 1, H, I, seed=12)
    rng = np.random.default_rng(7)
    lg = router_logits(T, layer_log_bias(1, E, 1.1, seed=0)[0], rng)
    ids, w = R.router_topk_softmax(lg, K)
    x = torch.from_numpy(rng.standard_normal((T, H)).astype(np.float32)).to(torch.bfloat16)
    dense = DenseExperts(pool)
    yr = R.moe_ffn(bf16_bits(x), ids, w, *dense.callables(),
                   shared=DenseExperts(shared).shared(0))
    return (pool.to(cuda_device), shared.to(cuda_device), x.to(cuda_device),
            torch.from_numpy(ids).to(cuda_device), torch.from_numpy(w).to(cuda_device), yr)


@pytest.mark.parametrize("kernel", ["fp4", "f16"])
def test_prefill_matches_oracle_at_prefill_config(cuda_device, prefill_case, kernel):
    pool, shared, x, ids, w, yr = prefill_case
    st = torch.full((1,), 77, dtype=torch.int32, device=cuda_device)
    y = ops.moe_ffn_prefill(pool, x, ids, w, shared=shared, status=st, kernel=kernel)
    y2 = ops.moe_ffn_prefill(pool, x, ids, w, shared=shared, kernel=kernel)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    assert torch.equal(y, y2)  # deterministic
    err = within(y, yr)
    assert err <= FFN_TOL, err
