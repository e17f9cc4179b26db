"""Seeded synthetic routing and activations with the benchmark shapes.

Routing skew follows the reference's synthetic trace generator (nvme-moe-bench/bench.py:232-264):
Zipf popularity p_r ~ r^-s over experts, a different random permutation per layer deciding which
expert gets which rank.  Router logits are N(0, 1) + ln p_e, so softmax top-k reproduces the
skew; tokens are N(0, 1) rounded to bf16.
"""
from __future__ import annotations

import numpy as np
import torch


def zipf_probs(n_experts: int, skew: float) -> np.ndarray:
    ranks = np.arange(1, n_experts + 1, dtype=np.float64)
    w = ranks ** (-skew)
    return w / w.sum()


def layer_log_bias(n_layers: int, n_experts: int, skew: float, seed: int = 0) -> np.ndarray:
    """[L, E] float32 ln p_e with a per-layer permutation of the Zipf ranks."""
    rng = np.random.default_rng(seed)
    base = zipf_probs(n_experts, skew)
    out = np.empty((n_layers, n_experts), np.float32)
    for layer in range(n_layers):
        perm = rng.permutation(n_experts)
        out[layer] = np.log(base[np.argsort(perm)]).astype(np.float32)
    return out


def router_logits(n_tok: int, bias: np.ndarray, rng: np.random.Generator) -> np.ndarray:
    return (rng.standard_normal((n_tok, bias.shape[-1])).astype(np.float32) + bias).astype(
        np.float32)


def tokens_bf16(n_tok: int, hidden: int, rng: np.random.Generator) -> torch.Tensor:
    return torch.from_numpy(rng.standard_normal((n_tok, hidden)).astype(np.float32)).to(
        torch.bfloat16)
