"""GPU parity of the block-scaled FP4 tensor-core FFN (NVFP4 pools) against the CPU oracle.

The oracle is the fp32 FFN over the dequantised weights and the bf16 activations; the kernel
feeds the weights unchanged to tcgen05 kind::mxf4nvf4 and the activations as 4 NVFP4 residual
terms, so the tolerance is the FFN one (max |y - ref| <= 1e-2 * max |ref|, mean <= 2e-3) and,
tighter, against the mma.sync kernel on the same inputs."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.formats import random_experts
from tests.test_gpu_kernels import _check_ffn, _oracle_ffn

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def fp4_kernel(monkeypatch):
    """These tests run the FP4 tensor-core kernel (selected per call by NVMOE_FFN_KERNEL)."""
    monkeypatch.setenv("NVMOE_FFN_KERNEL", "fp4")


def _case(dev, H, I, S, n_tok, k, shared, sgate, seed, x_scale=1.0):
    w = random_experts("nvfp4", S, H, I, seed=seed)
    sw = random_experts("nvfp4", 1, H, I, seed=500 + seed) if shared else None
    rng = np.random.default_rng(seed)
    x = torch.from_numpy((rng.standard_normal((n_tok, H)) * x_scale).astype(np.float32))
    x = x.to(torch.bfloat16)
    slots = np.stack([rng.choice(S, size=k, replace=False) for _ in range(n_tok)]).astype(np.int32)
    wts = rng.random((n_tok, k)).astype(np.float32)
    wts /= wts.sum(1, keepdims=True)
    g = (torch.from_numpy(rng.standard_normal(H).astype(np.float32) * 0.05).to(torch.bfloat16)
         if sgate else None)
    dargs = dict(pool=w.to(dev), x=x.to(dev), slot_ids=torch.from_numpy(slots).to(dev),
                 weights=torch.from_numpy(wts).to(dev),
                 shared=None if sw is None else sw.to(dev),
                 shared_gate=None if g is None else g.to(dev))
    return dargs, (w, x, slots, wts, sw, g)


@pytest.mark.parametrize("H,I,S,n_tok,k,shared,sgate", [
    (2048, 512, 128, 1, 10, True, False),
    (2048, 512, 128, 8, 10, True, True),
    (2048, 512, 128, 64, 10, True, False),
    (2048, 512, 40, 5, 8, False, False),
    (256, 256, 8, 1, 2, False, False),     # fewer units than CTAs
    (512, 256, 16, 3, 4, True, True),
    (4096, 1536, 24, 4, 8, True, False),   # GLM-shaped matrices
])
def test_fp4_ffn_matches_oracle(cuda_device, H, I, S, n_tok, k, shared, sgate):
    dargs, ref_args = _case(cuda_device, H, I, S, n_tok, k, shared, sgate, seed=H + n_tok)
    assert ops.ffn_path(dargs["pool"], dargs["x"], dargs["slot_ids"], dargs["weights"],
                        dargs["shared"]) == "fp4"
    y = ops.moe_ffn(**dargs)
    torch.cuda.synchronize()
    _check_ffn(y, _oracle_ffn(*ref_args))


@pytest.mark.parametrize("x_scale", [1e-3, 40.0, 900.0])
def test_fp4_ffn_activation_range(cuda_device, x_scale):
    """The 4-term activation split keeps its accuracy over a wide range of activation sizes."""
    dargs, ref_args = _case(cuda_device, 2048, 512, 32, 4, 8, True, False, seed=7,
                            x_scale=x_scale)
    y = ops.moe_ffn(**dargs)
    torch.cuda.synchronize()
    _check_ffn(y, _oracle_ffn(*ref_args))


def test_fp4_ffn_deterministic_and_close_to_mma_kernel(cuda_device, monkeypatch):
    dargs, _ = _case(cuda_device, 2048, 512, 64, 8, 10, True, True, seed=3)
    y1 = ops.moe_ffn(**dargs)
    y2 = ops.moe_ffn(**dargs)
    y3 = ops.moe_ffn(**dargs)
    torch.cuda.synchronize()
    assert torch.equal(y1, y2) and torch.equal(y1, y3)
    monkeypatch.setenv("NVMOE_FFN_KERNEL", "mma")
    assert ops.ffn_path(dargs["pool"], dargs["x"], dargs["slot_ids"], dargs["weights"],
                        dargs["shared"]) == "mma"
    ym = ops.moe_ffn(**dargs)
    torch.cuda.synchronize()
    a, b = y1.float(), ym.float()
    # two fp32 accumulations of the same products (bf16 outputs): a few bf16 ulps apart
    assert (a - b).abs().max().item() <= 4e-3 * b.abs().max().item()


def test_fp4_ffn_bad_slot_reports_status(cuda_device):
    H, I, S = 2048, 512, 8
    w = random_experts("nvfp4", S, H, I, seed=1).to(cuda_device)
    st = torch.zeros(1, dtype=torch.int32, device=cuda_device)
    ids = torch.tensor([[0, 1, 99]], dtype=torch.int32, device=cuda_device)
    x = torch.randn((1, H), device=cuda_device).to(torch.bfloat16)
    assert ops.ffn_path(w, x, ids, torch.ones((1, 3), device=cuda_device)) == "fp4"
    y = ops.moe_ffn(w, x, ids, torch.ones((1, 3), device=cuda_device), status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == -8
    assert torch.isfinite(y.float()).all()
