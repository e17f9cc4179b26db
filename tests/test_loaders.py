"""The on-disk expert formats that feed the host tier (nvmoe_b200/loaders.py): the FTW manifest
and shards of the Python engine (nvme_offload_cache.py:764-835) and the NVMOERPK interleaved
sidecar of the llama.cpp engine (scripts/moe_cache_probe.cpp:184-205, 788-800), written from
seeded pools and read back byte for byte, whole experts and straight into host-tier slots."""
import json
import os

import pytest
import torch

from nvmoe_b200 import loaders
from nvmoe_b200.formats import random_experts


def _same(a, b):
    return torch.equal(a.reshape(-1).view(torch.uint8), b.reshape(-1).view(torch.uint8))


def test_ftw_round_trip_across_shards(tmp_path):
    E, H, I = 12, 256, 128
    layers = [random_experts("nvfp4", E, H, I, seed=s) for s in (1, 2, 3)]
    loaders.write_ftw(str(tmp_path), layers, n_shards=4)
    man = json.loads((tmp_path / "freetoken_weight.json").read_text())
    assert len(man["shards"]) == 4 and len(man["tensors"]) == 3 * 6
    m = loaders.FtwModel(str(tmp_path))
    assert m.n_layers == 3 and m.n_experts == E
    ids = [7, 0, 11, 3]
    for li, w in enumerate(layers):
        got = m.experts(li, ids)
        idx = torch.tensor(ids)
        assert _same(got.gate_up.data, w.gate_up.data[idx])
        assert _same(got.gate_up.scale, w.gate_up.scale[idx])
        assert _same(got.gate_up.glob, w.gate_up.glob[idx])
        assert _same(got.down.data, w.down.data[idx])
        assert _same(got.down.scale, w.down.scale[idx])
        assert _same(got.down.glob, w.down.glob[idx])
        assert (got.hidden, got.inter) == (H, I)
    # straight into host-tier slots (bank order of FTW_BANKS)
    w = layers[2]
    host = [torch.zeros((4,) + tuple(t.shape[1:]), dtype=t.dtype) for t in
            (w.gate_up.data, w.gate_up.scale, w.gate_up.glob.reshape(-1, 1), w.down.data,
             w.down.scale, w.down.glob.reshape(-1, 1))]
    m.load_into(2, 9, host, 3)
    src = (w.gate_up.data, w.gate_up.scale, w.gate_up.glob.reshape(-1, 1), w.down.data,
           w.down.scale, w.down.glob.reshape(-1, 1))
    for h, s in zip(host, src):
        assert _same(h[3], s[9]) and not h[:3].any()
    # the host tier's own banks: global scales one fp32 per slot ([S], as the pools keep them)
    from nvmoe_b200.tier import _bank_tensors, _empty_like_slots
    tier_banks = _bank_tensors(_empty_like_slots(w, 5, pin=False))
    m.load_into(2, 4, tier_banks, 2)
    for h, s in zip(tier_banks, _bank_tensors(w)):
        assert _same(h[2], s[4])
    with pytest.raises(IndexError):
        m.read_row(0, "down_packed", E)
    m.close()


def test_ftw_missing_bank_is_reported(tmp_path):
    loaders.write_ftw(str(tmp_path), [random_experts("nvfp4", 4, 256, 128, seed=1)])
    p = tmp_path / "freetoken_weight.json"
    man = json.loads(p.read_text())
    man["tensors"] = [t for t in man["tensors"] if not t["name"].startswith("down_scale")]
    p.write_text(json.dumps(man))
    with pytest.raises(KeyError, match="down_scale#L00000"):
        loaders.FtwModel(str(tmp_path))


@pytest.mark.parametrize("quant", ["q2_k", "iq2_xxs"])
def test_interleaved_sidecar_round_trip(tmp_path, quant):
    E, H, I = 6, 512, 256
    layers = [random_experts(quant, E, H, I, seed=s) for s in (4, 5)]
    path = str(tmp_path / "interleaved_experts.bin")
    loaders.write_interleaved(path, layers)
    raw = open(path, "rb").read()
    assert int.from_bytes(raw[:8], "little") == loaders.RPK_MAGIC  # "NVMOERPK"
    s = loaders.InterleavedSidecar(path)
    assert (s.n_layers, s.n_experts) == (2, E)
    for li, (w, m) in enumerate(zip(layers, s.layers)):
        assert m.file_offset % 4096 == 0 and m.expert_size % 4096 == 0
        assert m.gate_row_bytes + m.up_row_bytes == w.gate_up.data[0].numel()
        for e in (0, E - 1, 2):
            g, u, d = s.read_expert(li, e)
            assert g + u == w.gate_up.data[e].numpy().tobytes()
            assert d == w.down.data[e].numpy().tobytes()
    w = layers[1]
    host = [torch.zeros((3,) + tuple(w.gate_up.data.shape[1:]), dtype=torch.uint8),
            torch.zeros((3,) + tuple(w.down.data.shape[1:]), dtype=torch.uint8)]
    s.load_into(1, 4, host, 1)
    assert torch.equal(host[0][1], w.gate_up.data[4]) and torch.equal(host[1][1], w.down.data[4])
    assert not host[0][0].any() and not host[1][2].any()
    s.close()


def test_interleaved_sidecar_rejects_other_files(tmp_path):
    p = tmp_path / "x.bin"
    p.write_bytes(b"\0" * 4096)
    with pytest.raises(ValueError, match="NVMOERPK"):
        loaders.InterleavedSidecar(str(p))
    p.write_bytes(b"\0" * 100)
    with pytest.raises(ValueError, match="4096"):
        loaders.InterleavedSidecar(str(p))


def test_sidecar_header_layout_is_the_packed_c_struct():
    # layer_meta: u64 + 5 x u32 packed = 28 bytes; the header's fixed part 24 bytes; 64 layers
    assert loaders._RPK_LAYER.size == 28 and loaders._RPK_HEAD.size == 24
    assert 24 + 64 * 28 <= loaders.RPK_HEADER_BYTES == 4096
