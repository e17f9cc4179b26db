"""Cache counters on the device (nvmoe_cache_stats_add): eval_cb's GPU-tier statistics
(scripts/moe_cache_probe.cpp:253-256; hits / misses per distinct id at :662-671, one callback per
call at :995), accumulated in stream order from the miss lists of remap calls, against the
oracle's hits and misses of the same Zipf-routed decode and prefill steps."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import ref_numpy as R
from oracle.native import OracleLayer

pytestmark = pytest.mark.gpu


def test_cache_stats_match_oracle_counts(cuda_device):
    E, k, S, n_tok, bpe = 512, 10, 128, 8, 1769480
    rng = np.random.default_rng(3)
    bias = layer_log_bias(1, E, 1.1, seed=5)[0]
    table = ops.SlotTableGPU(E, S, cuda_device)
    orc = OracleLayer(E, S)
    stats = ops.CacheStatsGPU(cuda_device)
    exp = dict.fromkeys(ops.STATS_FIELDS, 0)
    for st in range(40):
        decode = st % 5 != 0
        ids_np, _ = R.router_topk_softmax(router_logits(n_tok, bias, rng), k)
        ids = torch.from_numpy(ids_np).to(cuda_device)
        _, ml = ops.remap(table, ids, is_decode=decode)
        stats.add(ml, decode, bpe)
        ref = orc.eval(ids_np.reshape(-1), is_decode=decode)
        assert ref["status"] == 0
        nu, nm = len(ref["unique_ids"]), len(ref["miss_ids"])
        exp["calls"] += 1
        exp["gpu_hits"] += nu - nm
        exp["gpu_misses"] += nm
        exp["refill_bytes"] += nm * bpe
        if decode:
            exp["decode_calls"] += 1
            exp["decode_gpu_hits"] += nu - nm
            exp["decode_gpu_misses"] += nm
    # a call that fails (an id past the table) counts only as an error
    bad = torch.tensor([[1, E, 3]], dtype=torch.int32, device=cuda_device)
    _, ml = ops.remap(table, bad, True)
    stats.add(ml, True, bpe)
    exp["error_calls"] += 1
    got = stats.read()
    for f in ops.STATS_FIELDS:
        assert got[f] == exp[f], (f, got[f], exp[f])
    assert 0.0 < got["gpu_hit_rate"] < 1.0
    stats.reset()
    assert all(v == 0 for f, v in stats.read().items() if f in ops.STATS_FIELDS)
