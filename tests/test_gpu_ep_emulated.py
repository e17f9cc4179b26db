"""The CUDA expert-parallel stack (nvmoe_ep_dispatch -> pre-routed nvmoe_decode_layer ->
nvmoe_ep_combine, nvmoe_b200.ep.EPMoEStack) with 2 and 4 ranks held in one process on one GPU,
the all-to-alls done by segment copies (ep_forward_emulated): every rank's output is checked
against the oracle chain of the whole (unsharded) model, stage by stage on the GPU's own inputs:
  residual bit-exact; RMSNorm within 1 bf16 ulp (>= 99 % exact); gate logits |d| <= 1e-4 +
  1e-5 |ref|; the MoE output of each layer (routed experts on their owner ranks, shared expert
  on the home rank, summed over ranks) max |y - ref| <= 1e-2 max |ref|.
The decode shape is the Qwen3.8 layer (512 experts, top-10, H 2048, I 512, shared expert) with
128-slot pools per rank (all local experts resident from 4 ranks on) and a cold start for the
2-rank case (the pools start with the 64 most popular local experts, so misses are refilled)."""
import numpy as np
import pytest
import torch

from nvmoe_b200.engine import StackConfig
from nvmoe_b200.ep import EPMoEStack, ep_forward_emulated
from nvmoe_b200.formats import random_experts
from nvmoe_b200.synth import layer_log_bias
from oracle import ref_numpy as R
from tests.helpers import DenseExperts, bf16_bits, within

pytestmark = pytest.mark.gpu

E, K, H, I = 512, 10, 2048, 512


@pytest.mark.parametrize("world,batch,warm", [(2, 8, 64), (4, 5, 128)])
def test_ep_stack_matches_oracle(cuda_device, world, batch, warm):
    L = 2
    cfg = StackConfig(n_layers=L, n_experts=E, top_k=K, hidden=H, inter=I, cache_size=128)
    host = random_experts("nvfp4", E, H, I, seed=41)
    f = torch.from_numpy((2.0 ** (np.arange(E) % 5 - 2.0)).astype(np.float32))
    for m in (host.gate_up, host.down):
        m.glob.mul_(f)
    shared = random_experts("nvfp4", 1, H, I, seed=42)
    bias = layer_log_bias(L, E, 1.1, seed=3)
    ranking = np.argsort(-bias, axis=1, kind="stable")
    stacks = [EPMoEStack(cfg, batch, r, world, host, shared, device=cuda_device, seed=7 + r,
                         logit_bias=bias) for r in range(world)]
    per = E // world
    for st in stacks:
        lr = st.local_ranking(ranking)[:, :warm]
        st.local.prewarm(lr)
    dense = DenseExperts(host)
    sh = DenseExperts(shared).shared(0)
    W = bf16_bits(stacks[0].local.gate_w)
    gam = bf16_bits(stacks[0].local.norm_w)
    rng = np.random.default_rng(world)
    outs = [torch.empty((batch, H), dtype=torch.bfloat16, device=cuda_device) for _ in range(world)]
    for step in range(2):
        xs = [torch.from_numpy(rng.standard_normal((batch, H)).astype(np.float32)).to(
            torch.bfloat16).to(cuda_device) for _ in range(world)]
        ep_forward_emulated(stacks, xs, outs)
        torch.cuda.synchronize()
        for r, st in enumerate(stacks):
            assert int(st.status.item()) == 0
            h_in = bf16_bits(xs[r])
            for l in range(L):
                if l >= 1:
                    h_ref = R.residual_add_bf16(h_in, bf16_bits(st.y[l - 1]))
                    np.testing.assert_array_equal(bf16_bits(st.h[l]), h_ref)
                    h_in = h_ref
                xn = bf16_bits(st.xn[l])
                gap = np.abs(xn.astype(np.int32) - R.rmsnorm_bf16(h_in, gam[l], st.local.eps).astype(np.int32))
                assert gap.max() <= 1 and (gap == 0).mean() >= 0.99
                lg = st.logits[l].cpu().numpy()
                np.testing.assert_allclose(lg, R.router_gate_logits(xn, W[l], bias[l]),
                                           rtol=1e-5, atol=1e-4)
                rids, rw = R.router_topk_softmax(lg, K)
                yr = R.moe_ffn(xn, rids, rw, *dense.callables(), shared=sh)
                err = within(st.y[l], yr)
                assert err <= 1e-2, (step, r, l, err)
            np.testing.assert_array_equal(bf16_bits(outs[r]),
                                          R.residual_add_bf16(h_in, bf16_bits(st.y[L - 1])))
        for st in stacks:
            for p in st.plans:
                assert int(p.status.item()) == 0
