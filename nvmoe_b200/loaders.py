"""On-disk expert formats that feed the host tier.

FtwModel reads the Python engine's FTW layout: freetoken_weight.json lists shard files (each with
its offset in one global byte space) and one "experts_bank" tensor per (bank, layer) named
"<bank>#L<layer:05d>", shape [E, ...], whose row e is expert e (nvme_offload_cache.py:764-835;
banks gate_up_packed, gate_up_scale, gate_up_global, down_packed, down_scale, down_global,
:824-835).

InterleavedSidecar reads the llama.cpp engine's NVMOERPK file: a 4096-byte header (magic
0x4e564d4f4552504b, version 1, layer count, expert count, then per layer the file offset of
expert 0, the 4096-aligned bytes per expert and the gate / up / down row bytes;
scripts/moe_cache_probe.cpp:184-205, written by scripts/repack_unsloth_interleaved.cpp), then
each layer's experts back to back, expert e at file_offset + e * expert_size holding its gate,
up and down rows in that order (read at moe_cache_probe.cpp:788-800).

Both read one expert's rows straight into a host-tier slot (load_into), the reads the reference
issues to NVMe when the host tier misses.  The writers exist for tests and tooling.
"""
from __future__ import annotations

import bisect
import json
import os
import struct
from dataclasses import dataclass

import numpy as np
import torch

from .formats import ExpertWeights, QuantMatrix

FTW_BANKS = ("gate_up_packed", "gate_up_scale", "gate_up_global", "down_packed", "down_scale",
             "down_global")
_DTYPES = {"uint8": (np.uint8, torch.uint8), "float8_e4m3fn": (np.uint8, torch.uint8),
           "float16": (np.float16, torch.float16), "bfloat16": (np.uint16, torch.bfloat16),
           "float32": (np.float32, torch.float32)}


def _pread_exact(fd: int, n: int, off: int) -> bytes:
    out = bytearray()
    while len(out) < n:
        b = os.pread(fd, n - len(out), off + len(out))
        if not b:
            raise OSError(f"short read at offset {off + len(out)}")
        out += b
    return bytes(out)


@dataclass
class _BankLoc:
    fd: int
    offset: int      # of row 0 inside its shard
    row_bytes: int
    n_rows: int
    row_shape: tuple
    dtype: str


class FtwModel:
    """The expert banks of an FTW model directory (nvme_offload_cache.py:764-835)."""

    def __init__(self, model_dir: str):
        with open(os.path.join(model_dir, "freetoken_weight.json"), encoding="utf-8") as f:
            manifest = json.load(f)
        self.shards = sorted(manifest["shards"], key=lambda s: s["global_off"])
        starts = [s["global_off"] for s in self.shards]
        self.fds = {s["file"]: os.open(os.path.join(model_dir, s["file"]), os.O_RDONLY)
                    for s in self.shards}
        entries = {t["name"]: t for t in manifest["tensors"] if t["kind"] == "experts_bank"}
        layers = sorted({int(n.rsplit("#L", 1)[1]) for n in entries})
        self.n_layers = len(layers)
        self.loc: dict[tuple[int, str], _BankLoc] = {}
        for layer in layers:
            for bank in FTW_BANKS:
                name = f"{bank}#L{layer:05d}"
                e = entries.get(name)
                if e is None:
                    raise KeyError(f"FTW manifest missing expert entry {name}")
                i = bisect.bisect_right(starts, e["global_off"]) - 1
                if i < 0:
                    raise ValueError(f"{name} lies before the first shard")
                shard = self.shards[i]
                n_rows = e["shape"][0]
                self.loc[(layer, bank)] = _BankLoc(
                    self.fds[shard["file"]], e["global_off"] - shard["global_off"],
                    e["nbytes"] // n_rows, n_rows, tuple(e["shape"][1:]), e["dtype"])
        self.n_experts = self.loc[(layers[0], FTW_BANKS[0])].n_rows

    def close(self) -> None:
        for fd in getattr(self, "fds", {}).values():
            os.close(fd)
        self.fds = {}

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()

    def read_row(self, layer: int, bank: str, expert: int) -> bytes:
        lc = self.loc[(layer, bank)]
        if not 0 <= expert < lc.n_rows:
            raise IndexError(f"expert {expert} outside [0, {lc.n_rows})")
        return _pread_exact(lc.fd, lc.row_bytes, lc.offset + expert * lc.row_bytes)

    def load_into(self, layer: int, expert: int, dst: list[torch.Tensor], slot: int) -> None:
        """Expert `expert` of `layer` into host slot `slot` of the six FTW banks `dst` (the
        order of FTW_BANKS; CPU tensors, row `slot` contiguous)."""
        for bank, t in zip(FTW_BANKS, dst):
            row = t[slot]
            buf = self.read_row(layer, bank, expert)
            if row.numel() * row.element_size() != len(buf):
                raise ValueError(f"{bank}: host slot holds {row.numel() * row.element_size()} "
                                 f"bytes, the file's row {len(buf)}")
            row.reshape(-1).view(torch.uint8).copy_(torch.frombuffer(bytearray(buf),
                                                                     dtype=torch.uint8))

    def experts(self, layer: int, ids) -> ExpertWeights:
        """The NVFP4 experts `ids` of `layer` as a slot pool (slot i = ids[i]) on the CPU."""
        ids = list(ids)

        def bank(name):
            lc = self.loc[(layer, name)]
            npdt, tdt = _DTYPES[lc.dtype]
            rows = [np.frombuffer(self.read_row(layer, name, e), dtype=npdt) for e in ids]
            a = np.stack(rows).reshape((len(ids),) + lc.row_shape) if rows else \
                np.empty((0,) + lc.row_shape, npdt)
            return torch.from_numpy(a.copy()).view(tdt) if tdt == torch.bfloat16 else \
                torch.from_numpy(a.copy())
        gu, gus, gug = bank("gate_up_packed"), bank("gate_up_scale"), bank("gate_up_global")
        dn, dns, dng = bank("down_packed"), bank("down_scale"), bank("down_global")
        two_i, hidden = gu.shape[1], gu.shape[2] * 2
        inter = two_i // 2
        return ExpertWeights("nvfp4", hidden, inter,
                             QuantMatrix("nvfp4", two_i, hidden, gu, gus, gug.reshape(-1)),
                             QuantMatrix("nvfp4", hidden, inter, dn, dns, dng.reshape(-1)))


def write_ftw(model_dir: str, layers: list[ExpertWeights], n_shards: int = 2) -> None:
    """An FTW model directory holding `layers` (NVFP4 pools, slot e = expert e): the banks of
    every layer in FTW_BANKS order, split over n_shards files at bank boundaries."""
    os.makedirs(model_dir, exist_ok=True)
    blobs, tensors, off = [], [], 0
    for layer, w in enumerate(layers):
        arrays = [(w.gate_up.data, "uint8"), (w.gate_up.scale, "float8_e4m3fn"),
                  (w.gate_up.glob.reshape(-1, 1), "float32"), (w.down.data, "uint8"),
                  (w.down.scale, "float8_e4m3fn"), (w.down.glob.reshape(-1, 1), "float32")]
        for bank, (t, dt) in zip(FTW_BANKS, arrays):
            raw = t.contiguous().view(torch.uint8).numpy().tobytes()
            tensors.append({"name": f"{bank}#L{layer:05d}", "kind": "experts_bank",
                            "global_off": off, "shape": list(t.shape), "nbytes": len(raw),
                            "dtype": dt})
            blobs.append((off, raw))
            off += len(raw)
    per = max(1, -(-len(blobs) // n_shards))
    shards = []
    for i in range(0, len(blobs), per):
        part = blobs[i:i + per]
        name = f"experts-{len(shards):05d}.ftw"
        with open(os.path.join(model_dir, name), "wb") as f:
            for _, raw in part:
                f.write(raw)
        shards.append({"file": name, "global_off": part[0][0]})
    with open(os.path.join(model_dir, "freetoken_weight.json"), "w", encoding="utf-8") as f:
        json.dump({"shards": shards, "tensors": tensors}, f)


# ------------------------------------------------------------------ NVMOERPK sidecar
RPK_MAGIC = 0x4E564D4F4552504B   # "NVMOERPK"
RPK_VERSION = 1
RPK_MAX_LAYERS = 64
_RPK_HEAD = struct.Struct("<QIIII")          # magic, version, n_layers, n_experts, reserved
_RPK_LAYER = struct.Struct("<QIIIII")        # file_offset, expert_size, gate, up, down, pad
RPK_HEADER_BYTES = 4096
assert _RPK_HEAD.size + RPK_MAX_LAYERS * _RPK_LAYER.size <= RPK_HEADER_BYTES


@dataclass
class RpkLayer:
    file_offset: int
    expert_size: int
    gate_row_bytes: int
    up_row_bytes: int
    down_row_bytes: int
    pad_bytes: int


class InterleavedSidecar:
    """An NVMOERPK v1 file (moe_cache_probe.cpp:184-205): one read per expert."""

    def __init__(self, path: str):
        self.fd = os.open(path, os.O_RDONLY)
        try:
            hdr = _pread_exact(self.fd, RPK_HEADER_BYTES, 0)
        except OSError:
            self.close()
            raise ValueError(f"{path}: shorter than the 4096-byte NVMOERPK header") from None
        magic, version, n_layers, n_experts, _ = _RPK_HEAD.unpack_from(hdr, 0)
        if magic != RPK_MAGIC or version != RPK_VERSION or n_layers > RPK_MAX_LAYERS:
            self.close()
            raise ValueError(f"{path}: not an NVMOERPK v{RPK_VERSION} file")
        self.n_layers, self.n_experts = n_layers, n_experts
        self.layers = [RpkLayer(*_RPK_LAYER.unpack_from(hdr, _RPK_HEAD.size + i * _RPK_LAYER.size))
                       for i in range(n_layers)]

    def close(self) -> None:
        if getattr(self, "fd", -1) >= 0:
            os.close(self.fd)
            self.fd = -1

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        self.close()

    def read_expert(self, layer: int, expert: int) -> tuple[bytes, bytes, bytes]:
        """(gate, up, down) rows of one expert."""
        if not 0 <= expert < self.n_experts:
            raise IndexError(f"expert {expert} outside [0, {self.n_experts})")
        m = self.layers[layer]
        raw = _pread_exact(self.fd, m.expert_size, m.file_offset + expert * m.expert_size)
        g, u = m.gate_row_bytes, m.up_row_bytes
        return raw[:g], raw[g:g + u], raw[g + u:g + u + m.down_row_bytes]

    def load_into(self, layer: int, expert: int, dst: list[torch.Tensor], slot: int) -> None:
        """One expert into host slot `slot` of a pool's data banks: dst = [gate_up data
        [S, 2I, row], down data [S, H, row]] (gate rows then up rows, as the slot pools keep
        them)."""
        g, u, d = self.read_expert(layer, expert)
        for t, buf in ((dst[0], g + u), (dst[1], d)):
            row = t[slot]
            if row.numel() * row.element_size() != len(buf):
                raise ValueError(f"host slot holds {row.numel() * row.element_size()} bytes, "
                                 f"the file's rows {len(buf)}")
            row.reshape(-1).view(torch.uint8).copy_(torch.frombuffer(bytearray(buf),
                                                                     dtype=torch.uint8))


def write_interleaved(path: str, layers: list[ExpertWeights], align: int = 4096) -> None:
    """An NVMOERPK v1 file of `layers` (pools without separate scale banks, e.g. Q2_K or
    IQ2_XXS; slot e = expert e): per expert its gate, up and down rows, padded to `align`."""
    if len(layers) > RPK_MAX_LAYERS:
        raise ValueError(f"at most {RPK_MAX_LAYERS} layers")
    n_exp = layers[0].n_slots
    metas, off = [], RPK_HEADER_BYTES
    for w in layers:
        half = w.gate_up.data[0].numel() // 2
        dn = w.down.data[0].numel()
        size = -(-(2 * half + dn) // align) * align
        metas.append(RpkLayer(off, size, half, half, dn, size - 2 * half - dn))
        off += size * n_exp
    hdr = bytearray(RPK_HEADER_BYTES)
    _RPK_HEAD.pack_into(hdr, 0, RPK_MAGIC, RPK_VERSION, len(layers), n_exp, 0)
    for i, m in enumerate(metas):
        _RPK_LAYER.pack_into(hdr, _RPK_HEAD.size + i * _RPK_LAYER.size, m.file_offset,
                             m.expert_size, m.gate_row_bytes, m.up_row_bytes, m.down_row_bytes,
                             m.pad_bytes)
    with open(path, "wb") as f:
        f.write(hdr)
        for w, m in zip(layers, metas):
            gu = w.gate_up.data.contiguous().view(torch.uint8).reshape(n_exp, -1).numpy()
            dn = w.down.data.contiguous().view(torch.uint8).reshape(n_exp, -1).numpy()
            pad = bytes(m.pad_bytes)
            for e in range(n_exp):
                f.write(gu[e].tobytes())
                f.write(dn[e].tobytes())
                f.write(pad)
