"""The decode FFN (nvmoe_moe_ffn) on Q2_K and IQ2_XXS slot pools, with their in-register
fragment dequantisers, against the fp32 oracle on weights dequantised by ggml's rules
(oracle/ref_numpy.py), within the FFN tolerance.  Q2_K at the 48-layer stack's shape
(H 2048, I 512), IQ2_XXS at the GLM-shaped layer's (H 4096, I 1536)."""
import numpy as np
import pytest
import torch

from nvmoe_b200 import ops
from nvmoe_b200.formats import iq2xxs_grid, random_experts
from oracle import ref_numpy as R

pytestmark = pytest.mark.gpu


def _dense_fn(w, quant):
    H, I = w.hidden, w.inter
    grid = iq2xxs_grid() if quant == "iq2_xxs" else None
    cache = {}

    def get(which, s):
        if (which, s) in cache:
            return cache[(which, s)]
        m = w.gate_up if which != "down" else w.down
        rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
        blocks = m.data[s, rows].cpu().numpy()
        n_rows, K = blocks.shape[0], (H if which != "down" else I)
        v = R.dequant_q2_k(blocks) if quant == "q2_k" else R.dequant_iq2_xxs(blocks, grid)
        cache[(which, s)] = v.reshape(n_rows, K)
        return cache[(which, s)]
    return get


@pytest.mark.parametrize("quant,H,I,S,n_tok,k", [("q2_k", 2048, 512, 16, 1, 4),
                                                  ("q2_k", 2048, 512, 16, 5, 4),
                                                  ("iq2_xxs", 4096, 1536, 8, 3, 4)])
def test_ffn_gguf_formats_match_oracle(cuda_device, quant, H, I, S, n_tok, k):
    if quant == "iq2_xxs":
        ops.ensure_iq2xxs_grid(cuda_device)
    pool = random_experts(quant, S, H, I, seed=81).to(cuda_device)
    shared = random_experts(quant, 1, H, I, seed=82).to(cuda_device)
    rng = np.random.default_rng(83 + n_tok)
    x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(
        torch.bfloat16).to(cuda_device)
    ids = torch.from_numpy(np.stack([rng.choice(S, size=k, replace=False)
                                     for _ in range(n_tok)]).astype(np.int32)).to(cuda_device)
    w = torch.from_numpy(rng.random((n_tok, k)).astype(np.float32)).to(cuda_device)
    st = torch.full((1,), 77, dtype=torch.int32, device=cuda_device)
    y = ops.moe_ffn(pool, x, ids, w, shared=shared, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0
    d, ds = _dense_fn(pool, quant), _dense_fn(shared, quant)
    yr = R.moe_ffn(x.cpu().view(torch.int16).numpy().view(np.uint16), ids.cpu().numpy(),
                   w.cpu().numpy(), lambda s: d("gate", s), lambda s: d("up", s),
                   lambda s: d("down", s), shared=(ds("gate", 0), ds("up", 0), ds("down", 0)))
    yv = y.float().cpu().numpy()
    assert np.isfinite(yv).all()
    assert np.abs(yv - yr).max() <= 1e-2 * float(np.abs(yr).max())


@pytest.mark.parametrize("n_tok,k,shared", [(1, 4, False), (32, 4, False), (8, 4, True)])
def test_ffn_bf16_pool_matches_oracle(cuda_device, n_tok, k, shared):
    """bf16 slot pools (the CPU-plumbing layer: 64 experts, top-4, H 1024, I 256, 16 slots)
    through the decode FFN, which multiplies them in f16, against the fp32 oracle."""
    H, I, S = 1024, 256, 16
    pool = random_experts("bf16", S, H, I, seed=91).to(cuda_device)
    sh = random_experts("bf16", 1, H, I, seed=92).to(cuda_device) if shared else None
    rng = np.random.default_rng(93 + n_tok)
    x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(
        torch.bfloat16).to(cuda_device)
    ids = torch.from_numpy(np.stack([rng.choice(S, size=k, replace=False)
                                     for _ in range(n_tok)]).astype(np.int32)).to(cuda_device)
    w = torch.from_numpy(rng.random((n_tok, k)).astype(np.float32)).to(cuda_device)
    st = torch.full((1,), 77, dtype=torch.int32, device=cuda_device)
    y = ops.moe_ffn(pool, x, ids, w, shared=sh, status=st)
    torch.cuda.synchronize()
    assert int(st.item()) == 0

    def dense(wts):
        def get(which, s):
            m = wts.gate_up if which != "down" else wts.down
            rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
            b = m.data[s, rows].cpu().contiguous().view(torch.int16).numpy().view(np.uint16)
            return R.bf16_to_f32(b)
        return get
    d = dense(pool)
    shared_dense = None
    if shared:
        ds = dense(sh)
        shared_dense = (ds("gate", 0), ds("up", 0), ds("down", 0))
    yr = R.moe_ffn(x.cpu().view(torch.int16).numpy().view(np.uint16), ids.cpu().numpy(),
                   w.cpu().numpy(), lambda s: d("gate", s), lambda s: d("up", s),
                   lambda s: d("down", s), shared=shared_dense)
    yv = y.float().cpu().numpy()
    assert np.isfinite(yv).all()
    scale = float(np.abs(yr).max())
    assert np.abs(yv - yr).max() <= 1e-2 * scale
    assert np.abs(yv - yr).mean() <= 2e-3 * scale
