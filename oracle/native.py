"""ctypes access to the compiled oracle (test infrastructure only).

liboracle.so  — our C restatement of eval_cb's GPU + host tiers (oracle/remap_lru.c)
libref_slru.so — the reference's own SegmentedHostLru (scripts/segmented_host_lru.hpp) behind a
                 C shim, built from the reference tree by oracle/Makefile into oracle/_ref/
"""
from __future__ import annotations

import ctypes as C
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ORACLE_SO = HERE / "_build" / "liboracle.so"
REF_SLRU_SO = HERE / "_ref" / "libref_slru.so"
REF_SLRU_KAT = HERE / "_ref" / "test_segmented_host_lru"

_P = C.c_void_p
_I32P = np.ctypeslib.ndpointer(np.int32, flags="C_CONTIGUOUS")
_U32P = np.ctypeslib.ndpointer(np.uint32, flags="C_CONTIGUOUS")
_U8P = np.ctypeslib.ndpointer(np.uint8, flags="C_CONTIGUOUS")


def build() -> None:
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True)


def _load_oracle() -> C.CDLL:
    if not ORACLE_SO.exists():
        build()
    L = C.CDLL(str(ORACLE_SO))
    L.orc_layer_create.restype = _P
    L.orc_layer_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_double]
    L.orc_layer_destroy.argtypes = [_P]
    L.orc_layer_tables.argtypes = [_P, _I32P, _I32P, _U32P, _U32P]
    L.orc_layer_set_tables.argtypes = [_P, _I32P, _I32P, _U32P, C.c_uint32]
    L.orc_layer_host_tables.argtypes = [_P, _I32P, _I32P]
    L.orc_layer_eval.restype = C.c_int
    L.orc_layer_eval.argtypes = [_P, _I32P, C.c_int, C.c_int, C.c_int, _I32P, _I32P, _U8P, _I32P,
                                 _I32P, _I32P, _I32P, _I32P, _I32P, _I32P, _I32P, _I32P, _I32P,
                                 _I32P, _I32P]
    L.orc_slru_create.restype = _P
    L.orc_slru_create.argtypes = [C.c_int, C.c_double]
    L.orc_slru_destroy.argtypes = [_P]
    L.orc_slru_set_capacity_hint.argtypes = [_P, C.c_int64]
    L.orc_slru_insert_new.argtypes = [_P, C.c_int]
    L.orc_slru_touch.argtypes = [_P, C.c_int]
    L.orc_slru_contains.restype = C.c_int
    L.orc_slru_contains.argtypes = [_P, C.c_int]
    L.orc_slru_size.restype = C.c_int64
    L.orc_slru_size.argtypes = [_P]
    L.orc_slru_pop_lru.restype = C.c_int
    L.orc_slru_pop_lru.argtypes = [_P]
    L.orc_slru_pop_lru_excluding.restype = C.c_int
    L.orc_slru_pop_lru_excluding.argtypes = [_P, _I32P, C.c_int]
    L.orc_slru_discard.argtypes = [_P, C.c_int]
    return L


_oracle = None


def oracle_lib() -> C.CDLL:
    global _oracle
    if _oracle is None:
        _oracle = _load_oracle()
    return _oracle


class OracleLayer:
    """One layer of the llama.cpp engine's expert cache (GPU slots + optional host tier)."""

    def __init__(self, n_expert: int, cache_size: int, pinned_k: int = 0,
                 host_cache_size: int = 0, protected_ratio: float = 0.8):
        self.L = oracle_lib()
        self.n_expert, self.cache_size = n_expert, cache_size
        self.h = self.L.orc_layer_create(n_expert, cache_size, pinned_k, host_cache_size,
                                         protected_ratio)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.orc_layer_destroy(self.h)
            self.h = None

    def tables(self):
        a = np.empty(self.n_expert, np.int32)
        b = np.empty(self.cache_size, np.int32)
        c = np.empty(self.cache_size, np.uint32)
        d = np.empty(1, np.uint32)
        self.L.orc_layer_tables(self.h, a, b, c, d)
        return a, b, c, int(d[0])

    def set_tables(self, slot_of_real, real_in_slot, last_used, step):
        self.L.orc_layer_set_tables(self.h, np.ascontiguousarray(slot_of_real, np.int32),
                                    np.ascontiguousarray(real_in_slot, np.int32),
                                    np.ascontiguousarray(last_used, np.uint32), int(step))

    def eval(self, ids: np.ndarray, is_decode: bool, with_host: bool = False) -> dict:
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        n = ids.size
        cap = max(n, 1)
        out = np.empty(cap, np.int32)
        uid = np.empty(cap, np.int32)
        uhit = np.empty(cap, np.uint8)
        nu = np.zeros(1, np.int32)
        mid = np.empty(cap, np.int32)
        msl = np.empty(cap, np.int32)
        ev = np.empty(cap, np.int32)
        nm = np.zeros(1, np.int32)
        hg = np.empty(cap, np.int32)
        hh = np.empty(cap, np.int32)
        nh = np.zeros(1, np.int32)
        li = np.empty(cap, np.int32)
        lg = np.empty(cap, np.int32)
        lh = np.empty(cap, np.int32)
        nl = np.zeros(1, np.int32)
        rc = self.L.orc_layer_eval(self.h, ids, n, int(is_decode), int(with_host), out, uid, uhit,
                                   nu, mid, msl, ev, nm, hg, hh, nh, li, lg, lh, nl)
        u, m = int(nu[0]), int(nm[0])
        return {
            "status": rc,
            "slots": out[:n].copy(),
            "unique_ids": uid[:u].copy(),
            "unique_hit": uhit[:u].copy(),
            "miss_ids": mid[:m].copy(),
            "miss_slots": msl[:m].copy(),
            "evicted": ev[:m].copy(),
            "h2d": list(zip(hg[:int(nh[0])].tolist(), hh[:int(nh[0])].tolist())),
            "loads": list(zip(li[:int(nl[0])].tolist(), lg[:int(nl[0])].tolist(),
                              lh[:int(nl[0])].tolist())),
        }


class OracleSlru:
    def __init__(self, n_keys: int, ratio: float = 0.8):
        self.L = oracle_lib()
        self.h = self.L.orc_slru_create(n_keys, ratio)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.orc_slru_destroy(self.h)
            self.h = None

    def set_capacity_hint(self, c): self.L.orc_slru_set_capacity_hint(self.h, c)
    def insert_new(self, k): self.L.orc_slru_insert_new(self.h, k)
    def touch(self, k): self.L.orc_slru_touch(self.h, k)
    def contains(self, k): return bool(self.L.orc_slru_contains(self.h, k))
    def size(self): return int(self.L.orc_slru_size(self.h))
    def pop_lru(self): return int(self.L.orc_slru_pop_lru(self.h))

    def pop_lru_excluding(self, protect):
        p = np.ascontiguousarray(list(protect), np.int32)
        return int(self.L.orc_slru_pop_lru_excluding(self.h, p, p.size))

    def discard(self, k): self.L.orc_slru_discard(self.h, k)


class RefSlru:
    """The reference's own C++ SegmentedHostLru (compiled into oracle/_ref)."""

    _lib = None

    def __init__(self, ratio: float = 0.8):
        if RefSlru._lib is None:
            if not REF_SLRU_SO.exists():
                raise FileNotFoundError(str(REF_SLRU_SO))
            L = C.CDLL(str(REF_SLRU_SO))
            L.ref_slru_create.restype = _P
            L.ref_slru_create.argtypes = [C.c_double]
            L.ref_slru_destroy.argtypes = [_P]
            L.ref_slru_set_capacity_hint.argtypes = [_P, C.c_int64]
            L.ref_slru_insert_new.argtypes = [_P, C.c_int64]
            L.ref_slru_touch.argtypes = [_P, C.c_int64]
            L.ref_slru_contains.restype = C.c_int
            L.ref_slru_contains.argtypes = [_P, C.c_int64]
            L.ref_slru_size.restype = C.c_int64
            L.ref_slru_size.argtypes = [_P]
            L.ref_slru_pop_lru.restype = C.c_int64
            L.ref_slru_pop_lru.argtypes = [_P]
            L.ref_slru_pop_lru_excluding.restype = C.c_int64
            L.ref_slru_pop_lru_excluding.argtypes = [_P, np.ctypeslib.ndpointer(np.int64), C.c_int]
            L.ref_slru_discard.argtypes = [_P, C.c_int64]
            RefSlru._lib = L
        self.L = RefSlru._lib
        self.h = self.L.ref_slru_create(ratio)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ref_slru_destroy(self.h)
            self.h = None

    def set_capacity_hint(self, c): self.L.ref_slru_set_capacity_hint(self.h, c)
    def insert_new(self, k): self.L.ref_slru_insert_new(self.h, k)
    def touch(self, k): self.L.ref_slru_touch(self.h, k)
    def contains(self, k): return bool(self.L.ref_slru_contains(self.h, k))
    def size(self): return int(self.L.ref_slru_size(self.h))
    def pop_lru(self): return int(self.L.ref_slru_pop_lru(self.h))

    def pop_lru_excluding(self, protect):
        p = np.ascontiguousarray(list(protect), np.int64)
        return int(self.L.ref_slru_pop_lru_excluding(self.h, p, p.size))

    def discard(self, k): self.L.ref_slru_discard(self.h, k)


REF_EVALCB_SO = HERE / "_ref" / "libref_evalcb.so"


class RefEvalCb:
    """The reference's own eval_cb remap + host-tier block (scripts/moe_cache_probe.cpp:627-753,
    955-970) compiled into oracle/_ref/libref_evalcb.so by oracle/Makefile.  Same step interface
    as OracleLayer.eval; the reference always has a host tier (host_cache_size >= 1: give it
    n_expert slots to leave the GPU tier alone).  The reference aborts when a step has more
    distinct ids than slots: callers keep within the pool."""

    _lib = None

    def __init__(self, n_expert: int, cache_size: int, pinned_k: int = 0,
                 host_cache_size: int = 0, protected_ratio: float = 0.8):
        if host_cache_size < 1:
            raise ValueError("the reference's eval_cb always has a host tier (host_cache_size >= 1)")
        if RefEvalCb._lib is None:
            if not REF_EVALCB_SO.exists():
                raise FileNotFoundError(str(REF_EVALCB_SO))
            L = C.CDLL(str(REF_EVALCB_SO))
            L.ref_evalcb_create.restype = _P
            L.ref_evalcb_create.argtypes = [C.c_int, C.c_int, C.c_int, C.c_int, C.c_double]
            L.ref_evalcb_destroy.argtypes = [_P]
            L.ref_evalcb_step.restype = C.c_int
            L.ref_evalcb_step.argtypes = [_P, _I32P, C.c_int, C.c_int, C.c_int, _I32P, _I32P,
                                          _I32P, _I32P, _I32P, _I32P, _I32P, _I32P]
            L.ref_evalcb_tables.argtypes = [_P, _I32P, _I32P, _U32P, _U32P]
            RefEvalCb._lib = L
        self.L = RefEvalCb._lib
        self.n_expert, self.cache_size = n_expert, cache_size
        self.h = self.L.ref_evalcb_create(n_expert, cache_size, pinned_k, host_cache_size,
                                          protected_ratio)

    def __del__(self):
        if getattr(self, "h", None):
            self.L.ref_evalcb_destroy(self.h)
            self.h = None

    def eval(self, ids: np.ndarray, n_used: int, is_decode: bool) -> dict:
        ids = np.ascontiguousarray(ids, np.int32).reshape(-1)
        n = ids.size
        cap = max(n, 1)
        out = np.empty(cap, np.int32)
        hg, hh, nh = np.empty(cap, np.int32), np.empty(cap, np.int32), np.zeros(1, np.int32)
        li, lg, lh, nl = (np.empty(cap, np.int32), np.empty(cap, np.int32),
                          np.empty(cap, np.int32), np.zeros(1, np.int32))
        self.L.ref_evalcb_step(self.h, ids, n // n_used, n_used, int(is_decode), out, hg, hh, nh,
                               li, lg, lh, nl)
        return {"slots": out[:n].copy(),
                "h2d": list(zip(hg[:int(nh[0])].tolist(), hh[:int(nh[0])].tolist())),
                "loads": list(zip(li[:int(nl[0])].tolist(), lg[:int(nl[0])].tolist(),
                                  lh[:int(nl[0])].tolist()))}

    def tables(self):
        a = np.empty(self.n_expert, np.int32)
        b = np.empty(self.cache_size, np.int32)
        c = np.empty(self.cache_size, np.uint32)
        d = np.empty(1, np.uint32)
        self.L.ref_evalcb_tables(self.h, a, b, c, d)
        return a, b, c, int(d[0])


REF_PRUNE_SO = HERE / "_ref" / "libref_prune.so"


def ref_prune(ids, w, slot_of_real, host_slot_of_real, real_in_slot, nvme_thresh, host_thresh,
              min_keep, min_mass, is_decode=True):
    """The reference's own tail-pruning block (scripts/moe_cache_probe.cpp:523-625) compiled into
    oracle/_ref/libref_prune.so by oracle/Makefile; same interface as ref_numpy.prune_tail (the
    reference always has a host tier map: None becomes all -1)."""
    if not REF_PRUNE_SO.exists():
        raise FileNotFoundError(str(REF_PRUNE_SO))
    L = C.CDLL(str(REF_PRUNE_SO))
    fn = L.ref_prune
    fn.restype = None
    ids = np.ascontiguousarray(ids, np.int32).copy()
    w = np.ascontiguousarray(w, np.float32).copy()
    n, k = ids.shape
    sor = np.ascontiguousarray(slot_of_real, np.int32)
    hs = (np.full(len(sor), -1, np.int32) if host_slot_of_real is None
          else np.ascontiguousarray(host_slot_of_real, np.int32))
    ris = np.ascontiguousarray(real_in_slot, np.int32)
    pn, ph = C.c_long(0), C.c_long(0)
    fn(C.c_int(len(sor)), C.c_int(len(ris)), sor.ctypes.data_as(C.c_void_p),
       hs.ctypes.data_as(C.c_void_p), ris.ctypes.data_as(C.c_void_p),
       ids.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p), C.c_int(n), C.c_int(k),
       C.c_float(nvme_thresh), C.c_float(host_thresh), C.c_int(min_keep), C.c_float(min_mass),
       C.c_int(1 if is_decode else 0), C.byref(pn), C.byref(ph))
    return ids, w, pn.value, ph.value
