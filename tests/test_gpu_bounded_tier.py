"""The bounded host tier on the hot path (nvmoe_b200.tier.BoundedTierStack): per layer step the
GPU remap's miss list is read back, the native host tier (SLRU) places the misses, backing-store
loads fill pinned host slots and nvmoe_refill_async copies the misses into their GPU slots on a
side stream before the FFN.  Checked against the oracle's three-tier restatement of eval_cb
(oracle/remap_lru.c with its host tier): miss ids and slots, the host hits and their host slots,
the loads and their host slots, bit-exact; each layer's MoE output within
max |y - ref| <= 1e-2 max |ref| of the fp32 oracle on the backing store's experts."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import loaders
from nvmoe_b200.engine import StackConfig
from nvmoe_b200.formats import random_experts
from nvmoe_b200.synth import layer_log_bias
from nvmoe_b200.tier import BoundedTierStack
from oracle import ref_numpy as R
from oracle.native import OracleLayer
from tests.helpers import DenseExperts, bf16_bits, within

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("source", ["memory", "ftw_files"])
def test_bounded_host_tier_stack_matches_oracle(cuda_device, source, tmp_path):
    """source "ftw_files": host-tier misses are read from an FTW model directory on disk
    (loaders.FtwModel, every layer holding the same experts as the in-memory store)."""
    L, E, k, H, I, S, HS, B = 2, 64, 4, 2048, 512, 16, 24, 4
    cfg = StackConfig(n_layers=L, n_experts=E, top_k=k, hidden=H, inter=I, cache_size=S)
    backing = random_experts("nvfp4", E, H, I, seed=91)
    loader = None
    if source == "ftw_files":
        loaders.write_ftw(str(tmp_path), [backing] * L, n_shards=3)
        loader = loaders.FtwModel(str(tmp_path))
    stack = BoundedTierStack(cfg, HS, backing=backing, device=cuda_device, seed=91,
                             loader=loader)
    bias = layer_log_bias(L, E, 1.1, seed=6)
    stack.init_router(logit_bias=bias, seed=92)
    orc = [OracleLayer(E, S, host_cache_size=HS) for _ in range(L)]
    dense = DenseExperts(stack.backing)
    shared = [DenseExperts(stack.core.shared_all).shared(l) for l in range(L)]
    rng = np.random.default_rng(93)
    out = torch.empty((B, H), dtype=torch.bfloat16, device=cuda_device)
    n_load = n_hit = 0
    for step in range(8):
        x = torch.from_numpy(rng.standard_normal((B, H)).astype(np.float32)).to(
            torch.bfloat16).to(cuda_device)
        trace = []
        stack.forward(x, out, trace=trace)
        torch.cuda.synchronize()
        b = stack.buffers(B)
        for l in range(L):
            lg = b["logits"][l].cpu().numpy()
            rids, rw = R.router_topk_softmax(lg, k)
            f = orc[l].eval(rids.reshape(-1), is_decode=True, with_host=True)
            assert f["status"] == 0
            t = trace[l]
            np.testing.assert_array_equal(t["miss_ids"], f["miss_ids"])
            np.testing.assert_array_equal(t["miss_slots"], f["miss_slots"])
            h2d = [(int(t["miss_slots"][j]), int(t["host_slots"][j]))
                   for j in range(len(t["loads"])) if not t["loads"][j]]
            loads = [(int(t["miss_ids"][j]), int(t["miss_slots"][j]), int(t["host_slots"][j]))
                     for j in range(len(t["loads"])) if t["loads"][j]]
            assert h2d == list(f["h2d"]) and loads == list(f["loads"]), (step, l)
            n_load += len(loads)
            n_hit += len(h2d)
            np.testing.assert_array_equal(b["slots"][l].cpu().numpy().reshape(-1), f["slots"])
            yr = R.moe_ffn(bf16_bits(b["xn"][l]), rids, rw, *dense.callables(), shared=shared[l])
            assert within(b["y"][l], yr) <= 1e-2, (step, l)
    assert n_load > HS  # the host tier filled and evicted
    assert stack.stats["host_loads"] == n_load and stack.stats["host_hits"] == n_hit
