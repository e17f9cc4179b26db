"""R10 prefill (nvmoe_moe_ffn_prefill: token-sorted tcgen05 grouped GEMM, f16 and block-scaled
FP4 kernels) against the fp32 oracle on a small batch and on a batch whose slots span several
tiles, its determinism, and its bad-slot status."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.formats import random_experts
from oracle import ref_numpy as R

pytestmark = pytest.mark.gpu
H, I = 2048, 512


@pytest.fixture(autouse=True, params=["f16", "fp4"])
def prefill_kernel(request, monkeypatch):
    """Every test runs on both prefill kernels: block-scaled FP4 (the default) and tcgen05
    kind::f16 on weights dequantised into tensor memory (NVMOE_PREFILL_KERNEL=f16)."""
    monkeypatch.setenv("NVMOE_PREFILL_KERNEL", request.param)
    return request.param


def _dense(w, which, s):
    m = w.gate_up if which != "down" else w.down
    rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
    return R.dequant_nvfp4(m.data[s, rows].cpu().numpy(), m.scale[s, rows].cpu().numpy(),
                           m.glob[s].item())


def _inputs(rng, n_tok, k, S, skew, dev):
    p = np.arange(1, S + 1, dtype=np.float64) ** -skew
    p /= p.sum()
    ids = np.stack([rng.choice(S, size=k, replace=False, p=p) for _ in range(n_tok)]).astype(np.int32)
    w = rng.random((n_tok, k)).astype(np.float32)
    x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(torch.bfloat16)
    return x.to(dev), torch.from_numpy(ids).to(dev), torch.from_numpy(w).to(dev)


def test_prefill_matches_oracle_small(cuda_device):
    S, n_tok, k = 24, 80, 4
    pool = random_experts("nvfp4", S, H, I, seed=51).to(cuda_device)
    shared = random_experts("nvfp4", 1, H, I, seed=52).to(cuda_device)
    rng = np.random.default_rng(53)
    gate = torch.from_numpy((rng.standard_normal(H) * 0.02).astype(np.float32)).to(
        torch.bfloat16).to(cuda_device)
    x, ids, w = _inputs(rng, n_tok, k, S, 0.8, cuda_device)
    st = torch.full((1,), 77, dtype=torch.int32, device=cuda_device)
    y = ops.moe_ffn_prefill(pool, x, ids, w, shared=shared, shared_gate=gate, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    cache = {}

    def hd(which, s):
        if (which, s) not in cache:
            cache[(which, s)] = _dense(pool, which, s)
        return cache[(which, s)]
    sh = (_dense(shared, "gate", 0), _dense(shared, "up", 0), _dense(shared, "down", 0))
    yr = R.moe_ffn(x.cpu().view(torch.int16).numpy().view(np.uint16), ids.cpu().numpy(),
                   w.cpu().numpy(), lambda s: hd("gate", s), lambda s: hd("up", s),
                   lambda s: hd("down", s), shared=sh,
                   shared_gate_bf16=gate.cpu().view(torch.int16).numpy().view(np.uint16))
    yv = y.float().cpu().numpy()
    scale = float(np.abs(yr).max())
    assert np.abs(yv - yr).max() <= 1e-2 * scale


def test_prefill_matches_oracle_multi_tile(cuda_device):
    """1024 tokens over 64 slots with Zipf(1.1) skew: the hottest slots span several tiles."""
    from tests.helpers import DenseExperts, bf16_bits, within
    S, n_tok, k = 64, 1024, 10
    pool = random_experts("nvfp4", S, H, I, seed=61)
    shared = random_experts("nvfp4", 1, H, I, seed=62)
    rng = np.random.default_rng(63)
    x, ids, w = _inputs(rng, n_tok, k, S, 1.1, cuda_device)
    counts = np.bincount(ids.cpu().numpy().reshape(-1), minlength=S)
    assert counts.max() > 3 * 128  # the hottest slots span several tiles
    gp, gs = pool.to(cuda_device), shared.to(cuda_device)
    y = ops.moe_ffn_prefill(gp, x, ids, w, shared=gs)
    y2 = ops.moe_ffn_prefill(gp, x, ids, w, shared=gs)
    torch.cuda.synchronize()
    assert torch.equal(y, y2)  # deterministic
    yr = R.moe_ffn(bf16_bits(x), ids.cpu().numpy(), w.cpu().numpy(),
                   *DenseExperts(pool).callables(), shared=DenseExperts(shared).shared(0))
    assert within(y, yr) <= 1e-2


def test_prefill_reports_bad_slot(cuda_device):
    S, n_tok, k = 8, 16, 2
    pool = random_experts("nvfp4", S, H, I, seed=71).to(cuda_device)
    rng = np.random.default_rng(72)
    x, ids, w = _inputs(rng, n_tok, k, S, 0.0, cuda_device)
    ids[3, 1] = S + 5
    st = torch.zeros((1,), dtype=torch.int32, device=cuda_device)
    ops.moe_ffn_prefill(pool, x, ids, w, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == -8  # NVMOE_ERR_BAD_SLOT


def test_prefill_skips_empty_entries(cuda_device):
    """A negative slot id is an empty entry (the rows an expert-parallel rank receives carry
    the experts it does not own as -1): the result equals the oracle over the remaining entries,
    and a token without entries gets y = 0."""
    from tests.helpers import DenseExperts, bf16_bits, within
    S, n_tok, k = 24, 96, 5
    pool = random_experts("nvfp4", S, H, I, seed=81)
    rng = np.random.default_rng(82)
    x, ids, w = _inputs(rng, n_tok, k, S, 0.7, cuda_device)
    ids_h = ids.cpu().numpy()
    ids_h[rng.random(ids_h.shape) < 0.6] = -1
    ids_h[7, :] = -1
    ids = torch.from_numpy(ids_h).to(cuda_device)
    st = torch.full((1,), 77, dtype=torch.int32, device=cuda_device)
    y = ops.moe_ffn_prefill(pool.to(cuda_device), x, ids, w, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    # the oracle sees each empty entry as a zero-weight pick of an all-zero expert S (a slot of
    # its own, so a token's real picks are never merged with its empty ones)
    wh = w.cpu().numpy().copy()
    wh[ids_h < 0] = 0.0
    dense = DenseExperts(pool)
    zero = {"gate": np.zeros((I, H), np.float32), "up": np.zeros((I, H), np.float32),
            "down": np.zeros((H, I), np.float32)}
    pick = lambda which: (lambda s: zero[which] if s == S else dense.get(which, s))  # noqa: E731
    yr = R.moe_ffn(bf16_bits(x), np.where(ids_h < 0, S, ids_h), wh, pick("gate"), pick("up"),
                   pick("down"))
    assert within(y, yr) <= 1e-2
    assert not y[7].float().abs().any()
