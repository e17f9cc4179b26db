"""The native bounded host tier (nvmoe_host_tier_*, C++ in the library) against the oracle's
restatement of eval_cb's three tiers (oracle/remap_lru.c, moe_cache_probe.cpp:636-752), on CPU:
the oracle's GPU tier gives each step's distinct ids, hits and misses; the host tier's placement
of the misses (host hits and their slots, loads and their slots) and its maps must equal the
oracle's with its host tier enabled, over Zipf-routed steps with a host tier smaller than the
model."""
import numpy as np
import pytest

from nvmoe_b200.synth import layer_log_bias, router_logits
from nvmoe_b200.tier import HostTier
from oracle import ref_numpy as R
from oracle.native import OracleLayer


@pytest.mark.parametrize("E,S,HS,B,k", [(64, 16, 24, 4, 4), (512, 48, 96, 4, 10)])
def test_host_tier_matches_oracle(E, S, HS, B, k):
    gpu_only = OracleLayer(E, S)
    full = OracleLayer(E, S, host_cache_size=HS)
    tier = HostTier(E, HS)
    bias = layer_log_bias(1, E, 1.1, seed=E)[0]
    rng = np.random.default_rng(S)
    loads = hits = 0
    for step in range(120):
        ids, _ = R.router_topk_softmax(router_logits(B, bias, rng), k)
        g = gpu_only.eval(ids.reshape(-1), is_decode=True)
        f = full.eval(ids.reshape(-1), is_decode=True, with_host=True)
        assert g["status"] == 0 and f["status"] == 0
        np.testing.assert_array_equal(g["miss_ids"], f["miss_ids"])
        hs, ld = tier.resolve(g["unique_ids"], g["unique_hit"], g["miss_ids"])
        exp_h2d = [(gs, h) for gs, h in f["h2d"]]
        got_h2d = [(int(g["miss_slots"][j]), int(hs[j])) for j in range(len(hs)) if not ld[j]]
        assert got_h2d == exp_h2d, step
        exp_loads = [(i, gs, h) for i, gs, h in f["loads"]]
        got_loads = [(int(g["miss_ids"][j]), int(g["miss_slots"][j]), int(hs[j]))
                     for j in range(len(hs)) if ld[j]]
        assert got_loads == exp_loads, step
        loads += len(got_loads)
        hits += len(got_h2d)
    a, b = tier.tables()
    ea = np.empty(E, np.int32)
    eb = np.empty(HS, np.int32)
    full.L.orc_layer_host_tables(full.h, ea, eb)
    np.testing.assert_array_equal(a, ea)
    np.testing.assert_array_equal(b, eb)
    assert loads > HS and hits > 0  # the host tier filled up and then evicted
    # its counters are eval_cb's st->host_hits / st->host_misses (moe_cache_probe.cpp:727-734):
    # the oracle's host-to-slot copies and backing-store loads of the same steps
    assert tier.stats() == (hits, loads)
