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
