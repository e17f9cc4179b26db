"""Host tier (R4): the library's SLRU (C ABI, host code — no GPU needed) against the reference's
own Python traces, its C++ KATs restated, and random differential runs vs the reference C++."""
import ctypes
import json
from pathlib import Path

import numpy as np
import pytest

from nvmoe_b200 import _lib
from oracle import native

GOLD = Path(__file__).resolve().parent / "golden"


class ProductSlru:
    def __init__(self, ratio=0.8):
        self.L = _lib.lib()
        self.h = self.L.nvmoe_slru_create(ratio)
        assert self.h

    def __del__(self):
        if getattr(self, "h", None):
            self.L.nvmoe_slru_destroy(self.h)
            self.h = None

    def set_capacity_hint(self, c): self.L.nvmoe_slru_set_capacity_hint(self.h, c)
    def insert_new(self, k): self.L.nvmoe_slru_insert_new(self.h, k)
    def touch(self, k): self.L.nvmoe_slru_touch(self.h, k)
    def contains(self, k): return bool(self.L.nvmoe_slru_contains(self.h, k))
    def size(self): return int(self.L.nvmoe_slru_size(self.h))

    def pop_lru(self):
        k = ctypes.c_int64()
        rc = self.L.nvmoe_slru_pop_lru(self.h, ctypes.byref(k))
        return int(k.value) if rc == 0 else None

    def pop_lru_excluding(self, protect):
        p = (ctypes.c_int64 * max(1, len(protect)))(*protect)
        k = ctypes.c_int64()
        rc = self.L.nvmoe_slru_pop_lru_excluding(self.h, p, len(protect), ctypes.byref(k))
        return int(k.value) if rc == 0 else None

    def discard(self, k): self.L.nvmoe_slru_discard(self.h, k)


def test_reference_known_answers():
    """The 7 checks of scripts/test_segmented_host_lru.cpp:16-111, run on the product SLRU."""
    l = ProductSlru(); l.insert_new(1); l.insert_new(2)
    assert l.contains(1) and l.contains(2) and not l.contains(3) and l.size() == 2
    l = ProductSlru(); l.set_capacity_hint(10); l.insert_new(1); l.insert_new(2); l.touch(2)
    assert l.pop_lru() == 1
    l = ProductSlru(); l.set_capacity_hint(10); l.insert_new(5); l.touch(5); l.touch(5)
    assert l.contains(5) and l.size() == 1
    l = ProductSlru(0.5); l.set_capacity_hint(4)
    for k in (1, 2, 3):
        l.insert_new(k); l.touch(k)
    assert all(l.contains(k) for k in (1, 2, 3)) and l.pop_lru() == 1
    l = ProductSlru(); l.set_capacity_hint(10)
    for k in (10, 20, 30):
        l.insert_new(k)
    l.touch(20)
    assert [l.pop_lru(), l.pop_lru(), l.pop_lru()] == [10, 30, 20] and l.size() == 0
    l = ProductSlru(); l.set_capacity_hint(10); l.insert_new(7); l.touch(7); l.discard(7)
    assert not l.contains(7)
    l.discard(999)
    l = ProductSlru(); l.set_capacity_hint(100); l.set_capacity_hint(5)
    l.insert_new(1); l.touch(1)
    for i in range(2, 51):
        l.insert_new(i); l.touch(i)
    assert l.contains(1)
    assert ProductSlru().pop_lru() is None


def test_replays_reference_python_traces():
    from tests.test_oracle_pins import _replay
    for tr in json.loads((GOLD / "slru_traces.json").read_text()):
        _replay(ProductSlru(tr["ratio"]), tr["ops"])


@pytest.mark.parametrize("seed", range(6))
def test_differential_vs_reference_cpp(seed):
    if not native.REF_SLRU_SO.exists():
        pytest.skip("oracle/_ref not built (reference tree absent)")
    rng = np.random.default_rng(seed)
    ratio = float(rng.choice([0.8, 0.3, 1.0]))
    a, b = ProductSlru(ratio), native.RefSlru(ratio)
    n_keys = int(rng.integers(5, 200))
    present = set()
    for _ in range(3000):
        r = rng.random()
        if r < 0.02:
            c = int(rng.integers(1, 100)); a.set_capacity_hint(c); b.set_capacity_hint(c)
        elif r < 0.4:
            absent = [k for k in range(n_keys) if k not in present]
            if absent:
                k = int(rng.choice(absent)); a.insert_new(k); b.insert_new(k); present.add(k)
        elif r < 0.75:
            k = int(rng.integers(0, n_keys)); a.touch(k); b.touch(k)
        elif r < 0.85 and present:
            x, y = a.pop_lru(), b.pop_lru(); assert x == y; present.discard(x)
        elif r < 0.95 and present:
            prot = [int(v) for v in rng.choice(n_keys, size=min(n_keys, 8), replace=False)]
            x, y = a.pop_lru_excluding(prot), b.pop_lru_excluding(prot)
            assert x == y; present.discard(x)
        else:
            k = int(rng.integers(0, n_keys)); a.discard(k); b.discard(k); present.discard(k)
        assert a.size() == b.size()
