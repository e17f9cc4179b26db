"""Shared plumbing of the parity tests: dense fp32 expert weights from the oracle's dequantisers,
cached per expert, for checking the CUDA FFN against oracle/ref_numpy.moe_ffn."""
from __future__ import annotations

from collections import OrderedDict

import numpy as np
import torch

from oracle import ref_numpy as R


def dense_matrix(w, which: str, s: int) -> np.ndarray:
    """fp32 [rows, K] of slot s's gate / up / down in ExpertWeights w (NVFP4, CPU or GPU)."""
    I = w.inter
    m = w.gate_up if which != "down" else w.down
    rows = slice(0, I) if which == "gate" else (slice(I, 2 * I) if which == "up" else slice(None))
    return R.dequant_nvfp4_torch(m.data[s, rows].cpu(), m.scale[s, rows].cpu(),
                                 np.float32(m.glob[s].item())).numpy()


class DenseExperts:
    """Dense gate / up / down of the slots of an NVFP4 ExpertWeights, dequantised on first use
    and kept in a bounded LRU (a whole 512-expert layer in fp32 would take 6 GB)."""

    def __init__(self, w, capacity: int = 192):
        self.w, self.cap = w, capacity
        self.cache: OrderedDict = OrderedDict()

    def get(self, which: str, s: int) -> np.ndarray:
        key = (which, int(s))
        if key in self.cache:
            self.cache.move_to_end(key)
            return self.cache[key]
        v = dense_matrix(self.w, which, int(s))
        self.cache[key] = v
        if len(self.cache) > self.cap:
            self.cache.popitem(last=False)
        return v

    def callables(self):
        return (lambda s: self.get("gate", s), lambda s: self.get("up", s),
                lambda s: self.get("down", s))

    def shared(self, s: int = 0):
        return self.get("gate", s), self.get("up", s), self.get("down", s)


def bf16_bits(x: torch.Tensor) -> np.ndarray:
    return x.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def within(y: torch.Tensor, yr: np.ndarray, rel: float = 1e-2) -> float:
    """Max abs error of the CUDA output against the oracle, as a fraction of the oracle's
    largest magnitude (the FFN tolerance: max-abs within 1e-2 of max|ref|)."""
    yv = y.float().cpu().numpy()
    scale = float(np.abs(yr).max())
    return float(np.abs(yv - yr).max()) / max(scale, 1e-30)
