"""Slot-pool weight formats: synthetic generators and layout codecs.

Layouts (what the kernels read):
  NVFP4, FTW banks (nvme-moe-bench/nvme_offload_cache.py:824-835; performance.md:300-306):
      gate_up_packed [S, 2I, H/2] u8 (gate rows [0, I), up rows [I, 2I)), byte b holds
      w[2b] (low nibble) and w[2b+1] (high nibble) (scripts/convert_ftw_to_gguf.py:54-58);
      gate_up_scale [S, 2I, H/16] float8_e4m3fn; gate_up_global [S] fp32;
      down_packed [S, H, I/2]; down_scale [S, H, I/16]; down_global [S].
  GGUF block_nvfp4 (36 B / 64 values): 4 UE4M3 scales then 4 x 8 code bytes, byte j of
      sub-block k = (w[16k+j] low, w[16k+j+8] high) (convert_ftw_to_gguf.py:60-69).
  Q2_K (84 B / 256) and IQ2_XXS (66 B / 256): ggml super-blocks, rows of K/256 blocks.
  bf16: plain rows [S, rows, 2 K] u8 (the bf16 values), the CPU-plumbing layer's weights.

Synthetic distributions follow the benchmark configurations: E2M1 codes uniform over the 16
values, one E4M3 scale per 16 values drawn 2^U(-8,-2), fp32 global 1/448; Q2_K 2-bit quants,
4-bit scales and mins uniform, fp16 d, dmin ~ |N(0, 0.01)|; IQ2_XXS codebook indices, sign
indices and 4-bit scales uniform, fp16 d ~ |N(0, 0.01)|; bf16 weights ~ N(0, 0.02).
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np
import torch

NVFP4_GLOBAL = 1.0 / 448.0
Q2K_BLOCK_BYTES = 84
IQ2XXS_BLOCK_BYTES = 66


@dataclass
class QuantMatrix:
    """One matrix bank of a slot pool: data [S, rows, row_bytes] u8 (+ NVFP4 scales/global)."""
    quant: str                 # "nvfp4" | "q2_k" | "iq2_xxs" | "bf16"
    rows: int
    cols: int                  # K
    data: torch.Tensor         # u8 [S, rows, row_bytes]
    scale: torch.Tensor | None = None   # u8 (e4m3 bits) [S, rows, K/16]
    glob: torch.Tensor | None = None    # f32 [S]

    @property
    def n_slots(self) -> int:
        return self.data.shape[0]

    def to(self, device) -> "QuantMatrix":
        return QuantMatrix(self.quant, self.rows, self.cols, self.data.to(device),
                           None if self.scale is None else self.scale.to(device),
                           None if self.glob is None else self.glob.to(device))

    def slot(self, s: int) -> "QuantMatrix":
        return QuantMatrix(self.quant, self.rows, self.cols, self.data[s:s + 1],
                           None if self.scale is None else self.scale[s:s + 1],
                           None if self.glob is None else self.glob[s:s + 1])

    @property
    def bytes_per_slot(self) -> int:
        n = self.data[0].numel()
        if self.scale is not None:
            n += self.scale[0].numel()
        if self.glob is not None:
            n += 4
        return n


def row_bytes(quant: str, cols: int) -> int:
    if quant == "nvfp4":
        return cols // 2
    if quant == "q2_k":
        return cols // 256 * Q2K_BLOCK_BYTES
    if quant == "iq2_xxs":
        return cols // 256 * IQ2XXS_BLOCK_BYTES
    if quant == "bf16":
        return 2 * cols
    raise ValueError(quant)


def _fp16_abs_normal(shape, std, gen, device) -> torch.Tensor:
    v = torch.randn(shape, generator=gen, device=device, dtype=torch.float32).abs_() * std
    return v.to(torch.float16).view(torch.uint8).reshape(*shape, 2)


def random_matrix(quant: str, n_slots: int, rows: int, cols: int, gen: torch.Generator,
                  device="cpu") -> QuantMatrix:
    """Synthetic slot bank with the benchmark distributions (see module docstring)."""
    if quant == "nvfp4":
        assert cols % 16 == 0
        data = torch.randint(0, 256, (n_slots, rows, cols // 2), generator=gen, device=device,
                             dtype=torch.uint8)
        u = torch.rand((n_slots, rows, cols // 16), generator=gen, device=device) * 6.0 - 8.0
        scale = torch.exp2(u).to(torch.float8_e4m3fn).view(torch.uint8)
        glob = torch.full((n_slots,), NVFP4_GLOBAL, dtype=torch.float32, device=device)
        return QuantMatrix(quant, rows, cols, data, scale, glob)
    if quant == "q2_k":
        assert cols % 256 == 0
        nb = cols // 256
        body = torch.randint(0, 256, (n_slots, rows, nb, 80), generator=gen, device=device,
                             dtype=torch.uint8)
        d = _fp16_abs_normal((n_slots, rows, nb), 0.01, gen, device)
        dmin = _fp16_abs_normal((n_slots, rows, nb), 0.01, gen, device)
        data = torch.cat([body, d, dmin], dim=-1).reshape(n_slots, rows, nb * Q2K_BLOCK_BYTES)
        return QuantMatrix(quant, rows, cols, data.contiguous())
    if quant == "iq2_xxs":
        assert cols % 256 == 0
        nb = cols // 256
        d = _fp16_abs_normal((n_slots, rows, nb), 0.01, gen, device)
        body = torch.randint(0, 256, (n_slots, rows, nb, 64), generator=gen, device=device,
                             dtype=torch.uint8)
        data = torch.cat([d, body], dim=-1).reshape(n_slots, rows, nb * IQ2XXS_BLOCK_BYTES)
        return QuantMatrix(quant, rows, cols, data.contiguous())
    if quant == "bf16":  # the CPU-plumbing layer's weights: N(0, 0.02) in bf16
        w = torch.randn((n_slots, rows, cols), generator=gen, device=device) * 0.02
        data = w.to(torch.bfloat16).view(torch.uint8).reshape(n_slots, rows, 2 * cols)
        return QuantMatrix(quant, rows, cols, data.contiguous())
    raise ValueError(quant)


@dataclass
class ExpertWeights:
    """gate [S, I, H], up [S, I, H], down [S, H, I] of one slot pool.

    For NVFP4 gate and up are views of one FTW gate_up bank ([S, 2I, ...]) so the pool can be
    handed to the kernels exactly as the Python engine's bank_views() returns it."""
    quant: str
    hidden: int
    inter: int
    gate_up: QuantMatrix   # rows 2I: gate rows [0, I), up rows [I, 2I)
    down: QuantMatrix      # rows H

    @property
    def n_slots(self) -> int:
        return self.gate_up.n_slots

    @property
    def bytes_per_slot(self) -> int:
        return self.gate_up.bytes_per_slot + self.down.bytes_per_slot

    def to(self, device) -> "ExpertWeights":
        return ExpertWeights(self.quant, self.hidden, self.inter, self.gate_up.to(device),
                             self.down.to(device))

    def banks(self) -> tuple[torch.Tensor, ...]:
        """FTW bank order (gate_up_packed, gate_up_scale, gate_up_global, down_packed,
        down_scale, down_global) for NVFP4, (gate_up, down) for the GGUF formats and, as bf16
        tensors [S, 2I, H] / [S, H, I], for bf16."""
        if self.quant == "nvfp4":
            return (self.gate_up.data, self.gate_up.scale, self.gate_up.glob.view(-1, 1),
                    self.down.data, self.down.scale, self.down.glob.view(-1, 1))
        if self.quant == "bf16":
            return (self.gate_up.data.view(torch.bfloat16), self.down.data.view(torch.bfloat16))
        return (self.gate_up.data, self.down.data)


def random_experts(quant: str, n_slots: int, hidden: int, inter: int, seed: int = 0,
                   device="cpu") -> ExpertWeights:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    gu = random_matrix(quant, n_slots, 2 * inter, hidden, gen, device)
    dn = random_matrix(quant, n_slots, hidden, inter, gen, device)
    return ExpertWeights(quant, hidden, inter, gu, dn)


def select_experts(w: ExpertWeights, idx) -> ExpertWeights:
    """The experts idx (a sequence of slot indices) of w, copied in that order."""
    idx = torch.as_tensor(list(idx), dtype=torch.long, device=w.gate_up.data.device)

    def sel(m: QuantMatrix) -> QuantMatrix:
        return QuantMatrix(m.quant, m.rows, m.cols, m.data.index_select(0, idx).contiguous(),
                           None if m.scale is None else m.scale.index_select(0, idx).contiguous(),
                           None if m.glob is None else m.glob.index_select(0, idx).contiguous())
    return ExpertWeights(w.quant, w.hidden, w.inter, sel(w.gate_up), sel(w.down))


def concat_experts(a: ExpertWeights, b: ExpertWeights) -> ExpertWeights:
    """a's experts followed by b's (same format and shape)."""
    def cat(x: QuantMatrix, y: QuantMatrix) -> QuantMatrix:
        return QuantMatrix(x.quant, x.rows, x.cols, torch.cat([x.data, y.data]),
                           None if x.scale is None else torch.cat([x.scale, y.scale]),
                           None if x.glob is None else torch.cat([x.glob, y.glob]))
    return ExpertWeights(a.quant, a.hidden, a.inter, cat(a.gate_up, b.gate_up),
                         cat(a.down, b.down))


# ------------------------------------------------------------------ codecs
def ftw_to_gguf_nvfp4(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """FTW NVFP4 rows -> GGUF block_nvfp4 rows (scripts/convert_ftw_to_gguf.py:46-70):
    per 64 values 4 UE4M3 scale bytes (sign stripped) then 4 sub-blocks of 8 bytes with
    byte j = (w[j] low, w[j+8] high)."""
    codes = np.asarray(codes, np.uint8)
    scales = np.asarray(scales, np.uint8)
    *lead, nbytes = codes.shape
    nsub = scales.shape[-1]
    assert nbytes == nsub * 8 and nsub % 4 == 0
    w = codes.reshape(*lead, nsub, 8)
    vals = np.empty((*lead, nsub, 16), np.uint8)
    vals[..., 0::2] = w & 0x0F
    vals[..., 1::2] = w >> 4
    qs = (vals[..., :8] & 0x0F) | ((vals[..., 8:] & 0x0F) << 4)
    d = (scales & 0x7F).reshape(*lead, nsub // 4, 4)
    q = qs.reshape(*lead, nsub // 4, 32)
    return np.concatenate([d, q], axis=-1).reshape(*lead, nsub // 4 * 36)


def gguf_to_ftw_nvfp4(blocks: np.ndarray, n_cols: int) -> tuple[np.ndarray, np.ndarray]:
    """Inverse of ftw_to_gguf_nvfp4 (UE4M3 scales come back with a clear sign bit)."""
    b = np.asarray(blocks, np.uint8)
    *lead, nbytes = b.shape
    nsup = n_cols // 64
    assert nbytes == nsup * 36
    b = b.reshape(*lead, nsup, 36)
    d = b[..., :4].reshape(*lead, nsup * 4)
    qs = b[..., 4:].reshape(*lead, nsup * 4, 8)
    vals = np.concatenate([qs & 0x0F, qs >> 4], axis=-1)  # w[0..7], w[8..15]
    codes = (vals[..., 0::2] | (vals[..., 1::2] << 4)).reshape(*lead, nsup * 32)
    return codes.astype(np.uint8), d.astype(np.uint8)


def repack_nvfp4_pairs(blocks: np.ndarray) -> np.ndarray:
    """In-place order change of scripts/repack_nvfp4_gguf.cpp:97-116 applied to block_nvfp4
    rows: within each 8-byte sub-block the nibbles become (w[j], w[j+4]) pairs."""
    b = np.array(blocks, np.uint8, copy=True)
    *lead, nbytes = b.shape
    v = b.reshape(-1, 36)
    for k in range(4):
        p = v[:, 4 + 8 * k: 12 + 8 * k].copy()
        out = v[:, 4 + 8 * k: 12 + 8 * k]
        for i in range(4):
            out[:, 2 * i] = (p[:, i] & 0x0F) | ((p[:, i + 4] & 0x0F) << 4)
            out[:, 2 * i + 1] = (p[:, i] >> 4) | ((p[:, i + 4] >> 4) << 4)
    return b


def iq2xxs_grid() -> np.ndarray:
    """ggml's IQ2_XXS codebook (256 x 8 magnitudes in {8, 25, 43}) from the installed gguf-py."""
    from gguf.quants import IQ2_XXS  # ggml's table, shipped with gguf-py
    IQ2_XXS.init_grid()
    return np.asarray(IQ2_XXS.grid, np.float32).reshape(256, 8).astype(np.uint8)
