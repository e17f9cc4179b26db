"""The llama.cpp eval-callback binding compiled against include/nvmoe_b200.h and run from C++:
tests/evalcb/mock_eval_cb.cpp plays ggml_backend_sched with the callback the reference registers
(moe_cache_probe.cpp:439-997) over two chained MoE layers, the selected-experts view
non-contiguous (nb[1] = n_as_full * 4, test_sched_chain_shrink.cpp:75-105,211-215), layer 1's
tokens RMSNorm(x + y) of layer 0's.  Checked: the ids rewritten in place equal the oracle's
eval_cb slots, the columns outside the view are untouched, outputs are NaN-free (the reference
test's criterion, :314-322) and within the FFN tolerance of the fp32 oracle on each layer's GPU
input, which is itself checked against the oracle's RMSNorm (within 1 bf16 ulp)."""
import os
import shutil
import subprocess
from pathlib import Path

import numpy as np
import pytest

from nvmoe_b200.formats import random_experts
from oracle import ref_numpy as R
from oracle.native import OracleLayer
from tests.helpers import DenseExperts

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def test_mock_eval_cb_two_chained_layers(cuda_device, tmp_path):
    gxx = shutil.which("g++")
    if gxx is None:
        pytest.skip("g++ not available")
    exe = tmp_path / "mock_eval_cb"
    cuda = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda"))
    subprocess.run([gxx, "-std=c++17", "-O2", f"-I{ROOT / 'include'}", f"-I{cuda / 'include'}",
                    str(ROOT / "tests" / "evalcb" / "mock_eval_cb.cpp"), "-o", str(exe),
                    f"-L{ROOT / 'nvmoe_b200'}", "-lnvmoe_b200", f"-L{cuda / 'lib64'}", "-lcudart",
                    f"-Wl,-rpath,{ROOT / 'nvmoe_b200'}"], check=True)
    E, k, H, I, S, n_tok, n_as_full, NL = 64, 4, 2048, 512, 16, 4, 64, 2
    host = random_experts("nvfp4", E, H, I, seed=101)
    for name, t in (("gu_codes", host.gate_up.data), ("gu_scale", host.gate_up.scale),
                    ("gu_glob", host.gate_up.glob), ("dn_codes", host.down.data),
                    ("dn_scale", host.down.scale), ("dn_glob", host.down.glob)):
        t.contiguous().numpy().tofile(tmp_path / f"{name}.bin")
    rng = np.random.default_rng(102)
    # fixed distinct ids per token, as the reference test uses (e.g. {229,108,5,2,...})
    ids = np.stack([np.stack([rng.choice(E, size=k, replace=False) for _ in range(n_tok)])
                    for _ in range(NL)]).astype(np.int32)
    w = rng.random((NL, n_tok, k)).astype(np.float32)
    x = R.f32_to_bf16(rng.standard_normal((n_tok, H)).astype(np.float32))
    x.tofile(tmp_path / "x.bin")
    ids.tofile(tmp_path / "ids.bin")
    w.tofile(tmp_path / "w.bin")
    r = subprocess.run([str(exe), str(tmp_path), str(E), str(k), str(H), str(I), str(S),
                        str(n_tok), str(n_as_full), str(NL)], capture_output=True, text=True,
                       timeout=120)
    assert r.returncode == 0, r.stderr
    status = (tmp_path / "status.txt").read_text()
    assert status.startswith("OK ffn_status=0") and "untouched=1" in status, status
    y = np.fromfile(tmp_path / "y.bin", np.uint16).reshape(NL, n_tok, H)
    xin = np.fromfile(tmp_path / "xin.bin", np.uint16).reshape(NL, n_tok, H)
    slots = np.fromfile(tmp_path / "slots.bin", np.int32).reshape(NL, n_tok, k)
    dense = DenseExperts(host)
    np.testing.assert_array_equal(xin[0], x)
    for l in range(NL):
        if l > 0:
            xr = R.rmsnorm_bf16(R.residual_add_bf16(xin[l - 1], y[l - 1]),
                                np.full(H, 0x3F80, np.uint16), 1e-6)
            assert np.abs(xin[l].astype(np.int32) - xr.astype(np.int32)).max() <= 1
        x_in = xin[l]
        ref = OracleLayer(E, S).eval(ids[l].reshape(-1), is_decode=True)
        assert ref["status"] == 0
        np.testing.assert_array_equal(slots[l].reshape(-1), ref["slots"])
        yl = R.bf16_to_f32(y[l])
        assert np.isfinite(yl).all()
        yr = R.moe_ffn(x_in, ids[l], w[l], *dense.callables())
        assert np.abs(yl - yr).max() <= 1e-2 * float(np.abs(yr).max()), l
