"""Oracle parity of the dependent-layer stack (MoEStack.forward_chain): per layer the residual
add, RMSNorm and router gate GEMV (nvmoe_router_gate), then the decode layer step
(nvmoe_decode_layer waiting for the gate's logits), at the Qwen3.8 decode shape (512 experts,
top-10, H 2048, I 512, shared expert, 128 slots, a pool that starts without the 32 hottest
experts, distinct global scales per expert).

Each stage is checked against the oracle on the inputs the GPU stage itself received, so an
error cannot hide behind the previous stage's rounding:
  residual h_l = bf16(h_{l-1} + y_{l-1})       bit-exact
  RMSNorm x_l                                  within 1 bf16 ulp (summation order of mean(h^2)),
                                               >= 99 % of values bit-exact
  gate logits                                  |d| <= 1e-4 + 1e-5 |ref| (fp32 vs float64 sums)
  router ids / weights (of the GPU logits),
  slot ids, tables after the step              bit-exact / rtol 2e-6
  FFN output y_l                               max |y - ref| <= 1e-2 max |ref|
  final residual                               bit-exact
"""
import numpy as np
import pytest
import torch

from nvmoe_b200.engine import MoEStack, StackConfig
from nvmoe_b200.synth import layer_log_bias
from oracle import ref_numpy as R
from oracle.native import OracleLayer
from tests.helpers import DenseExperts, bf16_bits, within

pytestmark = pytest.mark.gpu

E, K, H, I, S = 512, 10, 2048, 512, 128


def _ulp_gap(a: np.ndarray, b: np.ndarray) -> np.ndarray:
    """Distance in bf16 ulps between two arrays of bf16 bit patterns of equal sign."""
    return np.abs(a.astype(np.int32) - b.astype(np.int32))


@pytest.mark.parametrize("batch", [1, 8, 20])
def test_dependent_stack_matches_oracle_stage_by_stage(cuda_device, batch):
    """(batch 20: the gate launch routes its three token blocks itself, fused top-k)"""
    L = 3
    stack = MoEStack(StackConfig(n_layers=L), device=cuda_device, seed=31)
    f = torch.from_numpy((2.0 ** (np.arange(E) % 5 - 2.0)).astype(np.float32))
    for m in (stack.host.gate_up, stack.host.down):
        m.glob.mul_(f)
    bias = layer_log_bias(L, E, 1.1, seed=2)
    warm = np.argsort(-bias, axis=1, kind="stable")[:, 32:32 + S]
    stack.prewarm(warm)
    stack.init_router(logit_bias=bias, seed=9)
    orc = []
    for l in range(L):
        o = OracleLayer(E, S)
        sor = np.full(E, -1, np.int32)
        sor[warm[l]] = np.arange(S, dtype=np.int32)
        o.set_tables(sor, warm[l].astype(np.int32), np.zeros(S, np.uint32), 0)
        orc.append(o)
    W = bf16_bits(stack.gate_w)
    gam = bf16_bits(stack.norm_w)
    dense = DenseExperts(stack.host)
    shared = [DenseExperts(stack.shared_all).shared(l) for l in range(L)]
    rng = np.random.default_rng(200 + batch)
    out = torch.empty((batch, H), dtype=torch.bfloat16, device=cuda_device)
    misses = 0
    for step in range(3):
        x = torch.from_numpy(rng.standard_normal((batch, H)).astype(np.float32)).to(
            torch.bfloat16)
        stack.forward_chain(x.to(cuda_device), out)
        torch.cuda.synchronize()
        b = stack.chain_buffers(batch)
        h_in = bf16_bits(x)  # residual entering layer 0
        for l in range(L):
            if l >= 1:
                h_ref = R.residual_add_bf16(h_in, bf16_bits(b["y"][l - 1]))
                np.testing.assert_array_equal(bf16_bits(b["h"][l]), h_ref)
                h_in = bf16_bits(b["h"][l])
            xn_gpu = bf16_bits(b["xn"][l])
            xn_ref = R.rmsnorm_bf16(h_in, gam[l], stack.eps)
            gap = _ulp_gap(xn_gpu, xn_ref)
            assert gap.max() <= 1 and (gap == 0).mean() >= 0.99, (step, l, gap.max())
            lg_gpu = b["logits"][l].cpu().numpy()
            lg_ref = R.router_gate_logits(xn_gpu, W[l], bias[l])
            np.testing.assert_allclose(lg_gpu, lg_ref, rtol=1e-5, atol=1e-4)
            rids, rw = R.router_topk_softmax(lg_gpu, K)
            ref = orc[l].eval(rids.reshape(-1), is_decode=True)
            plan = b["plans"][l]
            assert ref["status"] == 0 and int(plan.status.item()) == 0
            np.testing.assert_array_equal(plan.slot_ids.cpu().numpy().reshape(-1), ref["slots"])
            np.testing.assert_allclose(plan.weights.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
            sor, ris, lu, st = orc[l].tables()
            t = stack.tables[l]
            np.testing.assert_array_equal(t.slot_of_real.cpu().numpy(), sor)
            np.testing.assert_array_equal(t.real_in_slot.cpu().numpy(), ris)
            misses += len(ref["miss_ids"])
            yr = R.moe_ffn(xn_gpu, rids, rw, *dense.callables(), shared=shared[l])
            err = within(b["y"][l], yr)
            assert err <= 1e-2, (step, l, err)
        fin = R.residual_add_bf16(h_in, bf16_bits(b["y"][L - 1]))
        np.testing.assert_array_equal(bf16_bits(out), fin)
    assert misses > 0


def test_router_gate_norm_and_logits_match_oracle(cuda_device):
    """nvmoe_router_gate alone at the three supported widths and batches 1 / 8 / 64, with and
    without a residual delta, RMSNorm and logit bias."""
    from nvmoe_b200 import ops
    rng = np.random.default_rng(5)
    for Hh, Ee, n in ((1024, 64, 64), (2048, 512, 8), (4096, 288, 1)):
        resid = torch.from_numpy(rng.standard_normal((n, Hh)).astype(np.float32)).to(torch.bfloat16)
        delta = torch.from_numpy(rng.standard_normal((n, Hh)).astype(np.float32)).to(torch.bfloat16)
        wg = torch.from_numpy((rng.standard_normal((Ee, Hh)) / np.sqrt(Hh)).astype(np.float32)).to(
            torch.bfloat16)
        gm = torch.from_numpy((1 + 0.1 * rng.standard_normal(Hh)).astype(np.float32)).to(
            torch.bfloat16)
        lb = rng.standard_normal(Ee).astype(np.float32)
        for use_delta, use_norm, use_bias in ((True, True, True), (False, False, False)):
            d = cuda_device
            h, xo, lg = ops.router_gate(resid.to(d), wg.to(d),
                                        delta=delta.to(d) if use_delta else None,
                                        norm_weight=gm.to(d) if use_norm else None, eps=1e-6,
                                        logit_bias=torch.from_numpy(lb).to(d) if use_bias else None)
            torch.cuda.synchronize()
            h_ref = R.residual_add_bf16(bf16_bits(resid), bf16_bits(delta) if use_delta else None)
            np.testing.assert_array_equal(bf16_bits(h), h_ref)
            x_ref = R.rmsnorm_bf16(h_ref, bf16_bits(gm) if use_norm else None, 1e-6)
            gap = _ulp_gap(bf16_bits(xo), x_ref)
            assert gap.max() <= 1 and (gap == 0).mean() >= 0.99
            lg_ref = R.router_gate_logits(bf16_bits(xo), bf16_bits(wg), lb if use_bias else None)
            np.testing.assert_allclose(lg.cpu().numpy(), lg_ref, rtol=1e-5, atol=1e-4)
