"""The two GGUF-format decode configurations through the engine, against the oracle chain.

GLM-5.3-Flash-shaped layer (IQ2_XXS, 288 experts, sigmoid router with a selection bias and a
routed scaling factor, top-8, H 4096, I 1536, shared expert) through nvmoe_decode_layer with a
64-slot pool: router ids / weights, slot ids, tables after each step, FFN output.

Qwen3.8-shaped Q2_K stack of dependent layers (RMSNorm between layers, a pool of 25 % of the
512 experts per layer, misses refilled from the pinned host tier) through
MoEStack.forward_chain: each stage on the GPU's own inputs, as for the NVFP4 chain.

Tolerances: ids / slots / tables bit-exact, router weights rtol 2e-6, RMSNorm within 1 bf16 ulp,
logits |d| <= 1e-4 + 1e-5 |ref|, FFN outputs max |y - ref| <= 1e-2 max |ref|."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.engine import MoEStack, StackConfig
from nvmoe_b200.formats import iq2xxs_grid
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer
from tests.helpers import bf16_bits, within

pytestmark = pytest.mark.gpu


class _Dense:
    """Dense fp32 gate / up / down of a GGUF-format pool (ggml's dequantisers), in a bounded
    LRU (one GLM expert is 76 MB in fp32)."""

    def __init__(self, w, quant, capacity=48):
        from collections import OrderedDict
        self.w, self.quant, self.c, self.cap = w, quant, OrderedDict(), capacity
        self.grid = iq2xxs_grid() if quant == "iq2_xxs" else None

    def get(self, which, s):
        key = (which, int(s))
        if key in self.c:
            self.c.move_to_end(key)
        else:
            if len(self.c) >= self.cap:
                self.c.popitem(last=False)
            w, I, H = self.w, self.w.inter, self.w.hidden
            m = w.gate_up if which != "down" else w.down
            rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
            b = m.data[int(s), rows].cpu().numpy()
            K = H if which != "down" else I
            v = R.dequant_q2_k(b) if self.quant == "q2_k" else R.dequant_iq2_xxs(b, self.grid)
            self.c[key] = v.reshape(b.shape[0], K)
        return self.c[key]

    def fns(self):
        return (lambda s: self.get("gate", s), lambda s: self.get("up", s),
                lambda s: self.get("down", s))


def test_glm_iq2xxs_decode_layer_matches_oracle(cuda_device):
    E, k, H, I, S, B = 288, 8, 4096, 1536, 64, 3
    ops.ensure_iq2xxs_grid(cuda_device)
    cfg = StackConfig(n_layers=1, n_experts=E, top_k=k, hidden=H, inter=I, cache_size=S,
                      quant="iq2_xxs", router="sigmoid", routed_scaling=2.5)
    stack = MoEStack(cfg, device=cuda_device, seed=61)
    rng = np.random.default_rng(62)
    sel_bias = (0.1 * rng.standard_normal((1, E))).astype(np.float32)
    stack.set_router_bias(sel_bias)
    zipf = layer_log_bias(1, E, 1.0, seed=4)[0]
    orc = OracleLayer(E, S)
    dense = _Dense(stack.host, "iq2_xxs")
    sh = _Dense(stack.shared_all.to("cpu"), "iq2_xxs")
    shared = (sh.get("gate", 0), sh.get("up", 0), sh.get("down", 0))
    misses = 0
    for step in range(3):
        lg = router_logits(B, zipf, rng)
        x = torch.from_numpy(rng.standard_normal((B, H)).astype(np.float32)).to(torch.bfloat16)
        y = stack.layer_step(0, x.to(cuda_device), torch.from_numpy(lg).to(cuda_device))
        torch.cuda.synchronize()
        plan = stack.plans(B)[0]
        rids, rw, _ = R.router_topk_sigmoid_bias(lg, k, sel_bias[0], True, 2.5)
        ref = orc.eval(rids.reshape(-1), is_decode=True)
        assert ref["status"] == 0 and int(plan.status.item()) == 0
        np.testing.assert_array_equal(plan.slot_ids.cpu().numpy().reshape(-1), ref["slots"])
        np.testing.assert_allclose(plan.weights.cpu().numpy(), rw, rtol=2e-6, atol=1e-7)
        sor, ris, lu, st = orc.tables()
        np.testing.assert_array_equal(stack.tables[0].slot_of_real.cpu().numpy(), sor)
        np.testing.assert_array_equal(stack.tables[0].real_in_slot.cpu().numpy(), ris)
        misses += len(ref["miss_ids"])
        yr = R.moe_ffn(bf16_bits(x), rids, rw, *dense.fns(), shared=shared)
        assert within(y, yr) <= 1e-2, step
    assert misses > 0  # a cold pool: every first use is a refill from the host tier


def test_q2k_dependent_stack_matches_oracle(cuda_device):
    L, E, k, H, I, S, B = 2, 512, 10, 2048, 512, 128, 4
    cfg = StackConfig(n_layers=L, n_experts=E, top_k=k, hidden=H, inter=I, cache_size=S,
                      quant="q2_k")
    stack = MoEStack(cfg, device=cuda_device, seed=71)
    bias = layer_log_bias(L, E, 1.1, seed=5)
    warm = np.argsort(-bias, axis=1, kind="stable")[:, 16:16 + S]
    stack.prewarm(warm)
    stack.init_router(logit_bias=bias, seed=72)
    orc = []
    for l in range(L):
        o = OracleLayer(E, S)
        sor = np.full(E, -1, np.int32)
        sor[warm[l]] = np.arange(S, dtype=np.int32)
        o.set_tables(sor, warm[l].astype(np.int32), np.zeros(S, np.uint32), 0)
        orc.append(o)
    W, gam = bf16_bits(stack.gate_w), bf16_bits(stack.norm_w)
    dense = _Dense(stack.host, "q2_k")
    shared = []
    for l in range(L):
        d = _Dense(stack.shared_all.to("cpu"), "q2_k")
        shared.append((d.get("gate", l), d.get("up", l), d.get("down", l)))
    rng = np.random.default_rng(73)
    out = torch.empty((B, H), dtype=torch.bfloat16, device=cuda_device)
    misses = 0
    for step in range(2):
        x = torch.from_numpy(rng.standard_normal((B, H)).astype(np.float32)).to(torch.bfloat16)
        stack.forward_chain(x.to(cuda_device), out)
        torch.cuda.synchronize()
        b = stack.chain_buffers(B)
        h_in = bf16_bits(x)
        for l in range(L):
            if l >= 1:
                h_ref = R.residual_add_bf16(h_in, bf16_bits(b["y"][l - 1]))
                np.testing.assert_array_equal(bf16_bits(b["h"][l]), h_ref)
                h_in = h_ref
            xn = bf16_bits(b["xn"][l])
            gap = np.abs(xn.astype(np.int32) - R.rmsnorm_bf16(h_in, gam[l], stack.eps).astype(np.int32))
            assert gap.max() <= 1 and (gap == 0).mean() >= 0.99
            lg = b["logits"][l].cpu().numpy()
            np.testing.assert_allclose(lg, R.router_gate_logits(xn, W[l], bias[l]), rtol=1e-5,
                                       atol=1e-4)
            rids, rw = R.router_topk_softmax(lg, k)
            ref = orc[l].eval(rids.reshape(-1), is_decode=True)
            plan = b["plans"][l]
            assert ref["status"] == 0 and int(plan.status.item()) == 0
            np.testing.assert_array_equal(plan.slot_ids.cpu().numpy().reshape(-1), ref["slots"])
            misses += len(ref["miss_ids"])
            yr = R.moe_ffn(xn, rids, rw, *dense.fns(), shared=shared[l])
            assert within(b["y"][l], yr) <= 1e-2, (step, l)
        np.testing.assert_array_equal(bf16_bits(out), R.residual_add_bf16(h_in, bf16_bits(b["y"][L - 1])))
    assert misses > 0
