"""nvmoe_moe_ffn_noalloc: the FFN entry point for callers that cannot allocate device memory
while they run it (such as an eval callback inside another framework's memory management).

Called through the C ABI and compared with the regular nvmoe_moe_ffn on the same inputs, twice
in a row (the shared scratch array keeps the first call's contents), within the FFN tolerance
used by the other GPU tests.  This file is collected last on purpose."""
import ctypes as C

import numpy as np
import pytest
import torch

from nvmoe_b200 import _lib, ops
from nvmoe_b200.formats import random_experts

pytestmark = pytest.mark.gpu


def _args(pool_s, shared_s, x, ids, w, y):
    return _lib.FfnArgs(
        C.pointer(pool_s), C.pointer(shared_s) if shared_s is not None else None, None,
        x.data_ptr(), x.stride(0), ids.data_ptr(), ids.stride(0), w.data_ptr(), w.stride(0),
        ids.shape[1], x.shape[0], y.data_ptr(), y.stride(0), None, 0, None, 0)


def _within_tolerance(y, ref):
    y, ref = y.float().cpu().numpy(), ref.float().cpu().numpy()
    scale = float(np.abs(ref).max())
    assert scale > 0
    assert np.abs(y - ref).max() <= 1e-2 * scale


def test_noalloc_matches_regular_entry_point_on_two_calls(cuda_device):
    H, I, S = 2048, 512, 32
    pool = random_experts("nvfp4", S, H, I, seed=41).to(cuda_device)
    shared = random_experts("nvfp4", 1, H, I, seed=42).to(cuda_device)
    ps, ss = ops.expert_pool_struct(pool), ops.expert_pool_struct(shared)
    rng = np.random.default_rng(43)
    lib = _lib.lib()
    stream = torch.cuda.current_stream().cuda_stream
    for n_tok, k in ((8, 10), (3, 6)):  # two calls in a row, different shapes and inputs
        x = torch.from_numpy(rng.standard_normal((n_tok, H)).astype(np.float32)).to(
            torch.bfloat16).to(cuda_device)
        ids = torch.from_numpy(np.stack([rng.choice(S, size=k, replace=False)
                                         for _ in range(n_tok)]).astype(np.int32)).to(cuda_device)
        w = torch.from_numpy(rng.random((n_tok, k)).astype(np.float32)).to(cuda_device)
        y = torch.full((n_tok, H), float("nan"), dtype=torch.bfloat16, device=cuda_device)
        a = _args(ps, ss, x, ids, w, y)
        assert lib.nvmoe_moe_ffn_noalloc(C.byref(a), stream) == _lib.NVMOE_OK
        ref = ops.moe_ffn(pool, x, ids, w, shared=shared)
        torch.cuda.synchronize()
        _within_tolerance(y, ref)


def test_noalloc_rejects_calls_beyond_its_scratch(cuda_device):
    H, I, S = 2048, 512, 16
    pool = random_experts("nvfp4", S, H, I, seed=44).to(cuda_device)
    ps = ops.expert_pool_struct(pool)
    n_tok, k = 512, 10  # needs far more than the 16 MiB scratch
    assert ops.ffn_workspace_bytes(n_tok, k, H, I, S) > 16 << 20
    x = torch.zeros((n_tok, H), dtype=torch.bfloat16, device=cuda_device)
    ids = torch.zeros((n_tok, k), dtype=torch.int32, device=cuda_device)
    w = torch.zeros((n_tok, k), dtype=torch.float32, device=cuda_device)
    y = torch.full((n_tok, H), 7.0, dtype=torch.bfloat16, device=cuda_device)
    a = _args(ps, None, x, ids, w, y)
    rc = _lib.lib().nvmoe_moe_ffn_noalloc(C.byref(a), torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.NVMOE_ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert bool((y == 7.0).all())  # nothing was launched
