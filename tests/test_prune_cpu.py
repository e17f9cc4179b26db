"""(f)3 tail pruning (scripts/moe_cache_probe.cpp:523-625) on CPU: the oracle's restatement
against the reference's own block (compiled from the reference tree into oracle/_ref), and the
product's row function (nvmoe_b200/csrc/prune_device.cuh, the code the device kernel runs)
compiled for the host against the oracle; ids, weights and pruned counts bit for bit."""
import ctypes as C
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from oracle import ref_numpy as R
from oracle.native import REF_PRUNE_SO, ref_prune

HERE = Path(__file__).resolve().parent


def _case(seed):
    rng = np.random.default_rng(seed)
    E = int(rng.choice([64, 288, 512]))
    k = int(rng.choice([4, 8, 10]))
    S = int(rng.choice([16, 48, 128]))
    n = int(rng.choice([1, 3, 8, 32]))
    sor = np.full(E, -1, np.int32)
    ris = np.full(S, -1, np.int32)
    n_res = int(rng.integers(0, min(S, E) + 1))
    res = rng.choice(E, n_res, replace=False)
    slots = rng.choice(S, n_res, replace=False)
    sor[res] = slots
    ris[slots] = res
    hs = None
    if rng.random() < 0.7:
        hs = np.full(E, -1, np.int32)
        hres = rng.choice(E, int(rng.integers(0, E // 2)), replace=False)
        hs[hres] = np.arange(len(hres), dtype=np.int32)
    logits = rng.standard_normal((n, E)).astype(np.float32) * float(rng.choice([0.5, 1.0, 3.0]))
    ids, w = R.router_topk_softmax(logits, k)
    if rng.random() < 0.2:
        w = w * np.float32(rng.choice([1e-8, 3.0]))  # rows below the reference's 1e-6 total
    cfg = dict(nvme_thresh=float(rng.choice([0.0, 0.02, 0.08, 0.3])),
               host_thresh=float(rng.choice([0.0, 0.05, 0.2])),
               min_keep=int(rng.choice([1, 2, 4, 6])),
               min_mass=float(rng.choice([0.5, 0.8, 0.95])),
               is_decode=bool(rng.random() < 0.8))
    return (ids.astype(np.int32), w.astype(np.float32), sor, hs, ris), cfg


@pytest.mark.skipif(not REF_PRUNE_SO.exists(), reason="oracle/_ref not built (no reference tree)")
def test_oracle_matches_the_reference_block():
    pruned_any = 0
    for seed in range(300):
        (ids, w, sor, hs, ris), cfg = _case(seed)
        a = R.prune_tail(ids, w, sor, hs, ris, **cfg)
        b = ref_prune(ids, w, sor, hs, ris, **cfg)
        np.testing.assert_array_equal(a[0], b[0], err_msg=str(seed))
        assert a[1].tobytes() == b[1].tobytes(), seed
        assert a[2:] == b[2:], seed
        pruned_any += a[2] + a[3]
    assert pruned_any > 100  # the cases do prune


@pytest.fixture(scope="module")
def harness(tmp_path_factory):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    so = tmp_path_factory.mktemp("prune") / "libprune_host.so"
    subprocess.run([gxx, "-O2", "-std=c++17", "-ffp-contract=off", "-fPIC", "-shared",
                    str(HERE / "prune_host_harness.cpp"), "-o", str(so)], check=True)
    lib = C.CDLL(str(so))
    lib.prune_rows_host.restype = None
    return lib


def test_device_row_function_matches_oracle(harness):
    for seed in range(300, 600):
        (ids, w, sor, hs, ris), cfg = _case(seed)
        a = R.prune_tail(ids, w, sor, hs, ris, **cfg)
        gi, gw = ids.copy(), w.copy()
        cnt = np.zeros(2, np.int32)
        n, k = ids.shape
        harness.prune_rows_host(
            gi.ctypes.data_as(C.c_void_p), gw.ctypes.data_as(C.c_void_p), C.c_int(n), C.c_int(k),
            sor.ctypes.data_as(C.c_void_p),
            None if hs is None else hs.ctypes.data_as(C.c_void_p),
            ris.ctypes.data_as(C.c_void_p), C.c_int(len(ris)), C.c_int(len(sor)),
            C.c_float(cfg["nvme_thresh"]), C.c_float(cfg["host_thresh"]),
            C.c_float(cfg["min_mass"]), C.c_int(cfg["min_keep"]), C.c_int(int(cfg["is_decode"])),
            cnt.ctypes.data_as(C.c_void_p))
        np.testing.assert_array_equal(gi, a[0], err_msg=str(seed))
        assert gw.tobytes() == a[1].tobytes(), seed
        assert (int(cnt[0]), int(cnt[1])) == a[2:], seed
