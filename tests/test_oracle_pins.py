"""Pins the CPU oracle to the reference's own vectors and to gguf-py (CPU only)."""
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import native, ref_numpy as R

GOLD = Path(__file__).resolve().parent / "golden"


@pytest.fixture(scope="module")
def dq():
    return np.load(GOLD / "dequant_golden.npz")


def test_q2k_oracle_matches_gguf_golden(dq):
    np.testing.assert_array_equal(R.dequant_q2_k(dq["q2k_blocks"]).view(np.uint32),
                                  dq["q2k_values"].view(np.uint32))


def test_iq2xxs_oracle_matches_gguf_golden(dq):
    np.testing.assert_array_equal(R.ksigns(), dq["ksigns"])
    got = R.dequant_iq2_xxs(dq["iq2xxs_blocks"], dq["iq2xxs_grid"])
    np.testing.assert_array_equal(got.view(np.uint32), dq["iq2xxs_values"].view(np.uint32))


def test_nvfp4_oracle_matches_gguf_golden(dq):
    # gguf-py decodes block_nvfp4 (doubled kvalues x ue4m3 x 0.5); the FTW restatement must give
    # the same values bit for bit (scales here are positive, so the stripped sign is immaterial)
    got = R.dequant_nvfp4(dq["nvfp4_codes"], dq["nvfp4_scales"])
    np.testing.assert_array_equal(got.view(np.uint32), dq["nvfp4_values_noglobal"].view(np.uint32))


def test_dequant_oracle_matches_live_gguf():
    # the installed gguf-py is available here too: random blocks beyond the committed fixture
    gq = pytest.importorskip("gguf.quants")
    rng = np.random.default_rng(11)
    q2 = rng.integers(0, 256, size=(64, 84), dtype=np.uint8)
    q2[:, 80:84] = np.abs(rng.standard_normal((64, 2)) * 0.02).astype(np.float16).view(np.uint8)
    np.testing.assert_array_equal(R.dequant_q2_k(q2), gq.Q2_K.dequantize_blocks(q2.copy()).reshape(-1))
    iq = rng.integers(0, 256, size=(64, 66), dtype=np.uint8)
    iq[:, :2] = np.abs(rng.standard_normal((64, 1)) * 0.02).astype(np.float16).view(np.uint8)
    gq.IQ2_XXS.init_grid()
    grid = np.asarray(gq.IQ2_XXS.grid, np.float32).reshape(256, 8)
    np.testing.assert_array_equal(R.dequant_iq2_xxs(iq, grid),
                                  gq.IQ2_XXS.dequantize_blocks(iq.copy()).reshape(-1))


def test_router_oracle_reproduces_golden():
    g = np.load(GOLD / "router_golden.npz")
    ids, w = R.router_topk_softmax(g["softmax_logits"], 10)
    np.testing.assert_array_equal(ids, g["softmax_ids"])
    np.testing.assert_array_equal(w, g["softmax_w"])
    ids2, w2, _ = R.router_topk_sigmoid_bias(g["sigmoid_logits"], 8, g["sigmoid_bias"], True, 2.5)
    np.testing.assert_array_equal(ids2, g["sigmoid_ids"])
    np.testing.assert_array_equal(w2, g["sigmoid_w"])


def test_router_oracle_semantics():
    lg = np.array([[0.0, 3.0, 3.0, -1.0, 2.0]], np.float32)
    ids, w = R.router_topk_softmax(lg, 3)
    assert ids.tolist() == [[1, 2, 4]]  # tie at 3.0 -> lower id first
    e = np.exp(np.array([0.0, 0.0, -1.0], np.float32))
    np.testing.assert_allclose(w[0], e / e.sum(), rtol=1e-6)
    # GLM: choice uses score + bias, weights use the plain score
    ids2, w2, _ = R.router_topk_sigmoid_bias(np.zeros((1, 4), np.float32), 2,
                                             np.array([0, 1, 0, 2], np.float32), True, 1.0)
    assert ids2.tolist() == [[3, 1]]
    np.testing.assert_allclose(w2, [[0.5, 0.5]], rtol=1e-6)


def test_reference_slru_known_answer_tests_pass():
    """The reference's own SLRU KAT binary (scripts/test_segmented_host_lru.cpp), built by
    oracle/Makefile from the reference tree into oracle/_ref."""
    if not native.REF_SLRU_KAT.exists():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    r = subprocess.run([str(native.REF_SLRU_KAT)], capture_output=True, text=True)
    assert r.returncode == 0 and "all tests passed" in r.stdout


def _replay(lru, ops):
    for name, arg, expect in ops:
        if name == "hint":
            lru.set_capacity_hint(arg)
        elif name == "insert_new":
            lru.insert_new(arg)
        elif name == "touch":
            lru.touch(arg)
        elif name == "pop_lru":
            assert lru.pop_lru() == expect
        elif name == "pop_excluding":
            assert lru.pop_lru_excluding(arg) == expect
        elif name == "discard":
            lru.discard(arg)
        elif name == "contains":
            assert lru.contains(arg) == expect
        elif name == "size":
            assert lru.size() == expect


def test_oracle_slru_replays_reference_python_traces():
    import json
    traces = json.loads((GOLD / "slru_traces.json").read_text())
    for tr in traces:
        _replay(native.OracleSlru(tr["n_keys"], tr["ratio"]), tr["ops"])


def test_reference_cpp_slru_replays_reference_python_traces():
    """The reference's two SLRU implementations agree on the committed traces."""
    import json
    if not native.REF_SLRU_SO.exists():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    for tr in json.loads((GOLD / "slru_traces.json").read_text()):
        _replay(native.RefSlru(tr["ratio"]), tr["ops"])


def test_torch_nvfp4_dequant_equals_numpy_restatement():
    """The vectorised torch restatement used at full layer sizes gives the numpy restatement's
    values bit for bit (all codes, all E4M3 scale bytes incl. subnormals, a non-trivial global)."""
    rng = np.random.default_rng(123)
    codes = rng.integers(0, 256, size=(37, 64), dtype=np.uint8)
    scales = rng.integers(0, 256, size=(37, 8), dtype=np.uint8)
    scales[0, :] = np.arange(8, dtype=np.uint8)  # subnormals and zero
    a = R.dequant_nvfp4(codes, scales, np.float32(0.3125))
    b = R.dequant_nvfp4_torch(codes, scales, np.float32(0.3125)).numpy()
    assert a.shape == b.shape
    nan = np.isnan(a)
    np.testing.assert_array_equal(nan, np.isnan(b))  # scale bytes 0x7F / 0xFF (NaN payloads vary)
    np.testing.assert_array_equal(a[~nan].view(np.uint32), b[~nan].view(np.uint32))


@pytest.mark.parametrize("case", ["glm_a", "glm_b", "glm_c"])
def test_glm_router_oracle_matches_the_reference_router(case):
    """The oracle's sigmoid + selection-bias router against the reference's own GLM router
    (nvme_offload_cache.py:2980-3089, run by tests/golden/make_golden.py): the same experts in
    the same order; weights within 2e-6 relative (torch's row sum may add in another order)."""
    g = np.load(GOLD / "glm_router_golden.npz")
    E, k, n, norm = (int(v) for v in g[f"{case}_meta"])
    ids, w, _ = R.router_topk_sigmoid_bias(g[f"{case}_logits"], k, g[f"{case}_bias"],
                                           bool(norm), float(g[f"{case}_scale"][0]))
    np.testing.assert_array_equal(ids, g[f"{case}_ids"])
    np.testing.assert_allclose(w, g[f"{case}_w"], rtol=2e-6, atol=0)
