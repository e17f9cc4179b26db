"""Pins the eval_cb oracle (oracle/remap_lru.c, which every GPU remap test compares against) to the
reference itself: the reference's own remap + host-tier block of scripts/moe_cache_probe.cpp
(:627-753, :955-970), compiled from the reference tree by oracle/Makefile into oracle/_ref/.
Both run the same Zipf-routed steps; slot ids, tables and the host tier's h2d / load lists must
agree exactly, with and without pinned slots and a bounded host tier, and on the committed
golden traces (tests/golden/remap_traces.npz).  Skipped where oracle/_ref was not built."""
from pathlib import Path

import numpy as np
import pytest

from nvmoe_b200.synth import layer_log_bias, router_logits
from oracle import native, ref_numpy as R

GOLD = Path(__file__).resolve().parent / "golden"
pytestmark = pytest.mark.skipif(not native.REF_EVALCB_SO.exists(),
                                reason="oracle/_ref/libref_evalcb.so not built (no reference tree)")


@pytest.mark.parametrize("E,S,pinned,HS,B,k,decode",
                         [(64, 16, 0, 0, 3, 4, True), (64, 16, 4, 24, 3, 4, True),
                          (512, 128, 0, 200, 8, 10, True), (512, 128, 8, 0, 8, 10, False),
                          (288, 64, 0, 96, 4, 8, True)])
def test_oracle_equals_reference_evalcb(E, S, pinned, HS, B, k, decode):
    ours = native.OracleLayer(E, S, pinned_k=pinned, host_cache_size=HS)
    # the reference always runs with a host tier (an empty one would pop an empty LRU); for the
    # GPU tier alone it gets one holding every expert, which never evicts
    ref = native.RefEvalCb(E, S, pinned_k=pinned, host_cache_size=HS if HS > 0 else E)
    bias = layer_log_bias(1, E, 1.1, seed=E + S)[0]
    rng = np.random.default_rng(E * S)
    for step in range(150):
        ids, _ = R.router_topk_softmax(router_logits(B, bias, rng), k)
        if len(np.unique(ids)) > S:
            continue  # the reference aborts: the ubatch clamp keeps real steps below this
        a = ours.eval(ids.reshape(-1), is_decode=decode, with_host=HS > 0)
        b = ref.eval(ids.reshape(-1), k, is_decode=decode)
        assert a["status"] == 0
        np.testing.assert_array_equal(a["slots"], b["slots"], err_msg=f"step {step}")
        if HS > 0:
            assert a["h2d"] == b["h2d"] and a["loads"] == b["loads"], step
    for x, y in zip(ours.tables(), ref.tables()):
        np.testing.assert_array_equal(np.asarray(x), np.asarray(y))


def test_golden_remap_traces_replay_through_reference():
    g = np.load(GOLD / "remap_traces.npz")
    names = sorted({k[:-len("_meta")] for k in g.files if k.endswith("_meta")})
    assert names
    for name in names:
        E, k, S, pinned, n_tok, steps = (int(v) for v in g[f"{name}_meta"])
        ref = native.RefEvalCb(E, S, pinned_k=pinned, host_cache_size=E)
        ids, slots = g[f"{name}_ids"], g[f"{name}_slots"]
        for i in range(steps):
            out = ref.eval(ids[i].reshape(-1), k, is_decode=True)
            np.testing.assert_array_equal(out["slots"], slots[i].reshape(-1), err_msg=f"{name} {i}")
