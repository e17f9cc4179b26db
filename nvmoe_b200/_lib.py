"""ctypes binding of libnvmoe_b200.so (include/nvmoe_b200.h).

The library is the product: there is no fallback.  `lib()` raises if the shared object has not
been built (``python -m nvmoe_b200.build``) or fails to load.
"""
from __future__ import annotations

import ctypes as C
import threading
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libnvmoe_b200.so"

NVMOE_OK = 0
NVMOE_ERR_INVALID_ARG = -1
NVMOE_ERR_BAD_EXPERT_ID = -2
NVMOE_ERR_CACHE_OVERFLOW = -3
NVMOE_ERR_CUDA = -4
NVMOE_ERR_WORKSPACE = -5
NVMOE_ERR_UNSUPPORTED = -6
NVMOE_ERR_HOST_LOAD = -7
NVMOE_ERR_BAD_SLOT = -8
NVMOE_ERR_NO_TABLES = -9
NVMOE_ERR_TIMEOUT = -10
NVMOE_ERR_SCRATCH_LIMIT = -11
NVMOE_ERR_GROUP_LIMIT = -12

STATUS_NAMES = {
    0: "NVMOE_OK",
    -1: "NVMOE_ERR_INVALID_ARG",
    -2: "NVMOE_ERR_BAD_EXPERT_ID",
    -3: "NVMOE_ERR_CACHE_OVERFLOW",
    -4: "NVMOE_ERR_CUDA",
    -5: "NVMOE_ERR_WORKSPACE",
    -6: "NVMOE_ERR_UNSUPPORTED",
    -7: "NVMOE_ERR_HOST_LOAD",
    -8: "NVMOE_ERR_BAD_SLOT",
    -9: "NVMOE_ERR_NO_TABLES",
    -10: "NVMOE_ERR_TIMEOUT",
    -11: "NVMOE_ERR_SCRATCH_LIMIT",
    -12: "NVMOE_ERR_GROUP_LIMIT",
}

NVMOE_Q_NVFP4 = 0
NVMOE_Q_Q2_K = 1
NVMOE_Q_IQ2_XXS = 2
NVMOE_Q_BF16 = 3

NVMOE_ROUTER_SOFTMAX = 0
NVMOE_ROUTER_SIGMOID_BIAS = 1

NVMOE_KERNEL_DEFAULT = 0
NVMOE_KERNEL_MMA = 1
NVMOE_KERNEL_FP4 = 2
NVMOE_KERNEL_F16 = 3


class NvmoeError(RuntimeError):
    def __init__(self, status: int, where: str, detail: str = ""):
        self.status = status
        name = STATUS_NAMES.get(status, str(status))
        super().__init__(f"{where}: {name}{(' — ' + detail) if detail else ''}")


class SlotTable(C.Structure):
    _fields_ = [
        ("slot_of_real", C.c_void_p),
        ("real_in_slot", C.c_void_p),
        ("slot_last_used", C.c_void_p),
        ("current_step", C.c_void_p),
        ("n_expert", C.c_int32),
        ("cache_size", C.c_int32),
        ("pinned_k", C.c_int32),
        ("id_base", C.c_int32),
    ]


class MissList(C.Structure):
    _fields_ = [
        ("unique_ids", C.c_void_p),
        ("unique_slot", C.c_void_p),
        ("unique_hit", C.c_void_p),
        ("miss_ids", C.c_void_p),
        ("miss_slots", C.c_void_p),
        ("evicted_ids", C.c_void_p),
        ("counts", C.c_void_p),
        ("capacity", C.c_int32),
    ]


class MatrixBank(C.Structure):
    _fields_ = [
        ("data", C.c_void_p),
        ("slot_stride", C.c_int64),
        ("row_stride", C.c_int64),
        ("scale", C.c_void_p),
        ("scale_slot_stride", C.c_int64),
        ("scale_row_stride", C.c_int64),
        ("global_scale", C.c_void_p),
        ("global_stride", C.c_int64),
    ]


class ExpertPool(C.Structure):
    _fields_ = [
        ("quant", C.c_int32),
        ("hidden", C.c_int32),
        ("inter", C.c_int32),
        ("n_slots", C.c_int32),
        ("gate", MatrixBank),
        ("up", MatrixBank),
        ("down", MatrixBank),
    ]


class FfnArgs(C.Structure):
    _fields_ = [
        ("pool", C.POINTER(ExpertPool)),
        ("shared", C.POINTER(ExpertPool)),
        ("shared_gate", C.c_void_p),
        ("x", C.c_void_p),
        ("x_row_stride", C.c_int64),
        ("slot_ids", C.c_void_p),
        ("ids_row_stride", C.c_int64),
        ("weights", C.c_void_p),
        ("weights_row_stride", C.c_int64),
        ("top_k", C.c_int32),
        ("n_tok", C.c_int32),
        ("y", C.c_void_p),
        ("y_row_stride", C.c_int64),
        ("workspace", C.c_void_p),
        ("workspace_bytes", C.c_size_t),
        ("status", C.c_void_p),
        ("kernel", C.c_int32),
    ]


class RefillBank(C.Structure):
    _fields_ = [
        ("dst", C.c_void_p),
        ("src", C.c_void_p),
        ("dst_slot_stride", C.c_int64),
        ("src_slot_stride", C.c_int64),
        ("row_bytes", C.c_int64),
    ]


class DecodeArgs(C.Structure):
    _fields_ = [
        ("logits", C.c_void_p),
        ("logits_row_stride", C.c_int64),
        ("router_mode", C.c_int32),
        ("router_bias", C.c_void_p),
        ("norm_topk", C.c_int32),
        ("routed_scaling", C.c_float),
        ("top_k", C.c_int32),
        ("n_tok", C.c_int32),
        ("is_decode", C.c_int32),
        ("table", SlotTable),
        ("misses", MissList),
        ("slot_ids", C.c_void_p),
        ("weights", C.c_void_p),
        ("refill_banks", C.POINTER(RefillBank)),
        ("n_refill_banks", C.c_int32),
        ("host_slot_of_id", C.c_void_p),
        ("ffn", FfnArgs),
        ("early_outputs", C.c_int32),
        ("inputs_after_wait", C.c_int32),
        ("routed_ids", C.c_void_p),
        ("routed_weights", C.c_void_p),
        ("routed_row_stride", C.c_int64),
    ]


class EpDispatchArgs(C.Structure):
    _fields_ = [
        ("x", C.c_void_p),
        ("x_row_stride", C.c_int64),
        ("ids", C.c_void_p),
        ("weights", C.c_void_p),
        ("shared_gate", C.c_void_p),
        ("with_shared", C.c_int32),
        ("n_tok", C.c_int32),
        ("top_k", C.c_int32),
        ("hidden", C.c_int32),
        ("n_expert", C.c_int32),
        ("world", C.c_int32),
        ("rank", C.c_int32),
        ("send", C.c_void_p),
        ("slot_of", C.c_void_p),
        ("status", C.c_void_p),
    ]


class EpCombineArgs(C.Structure):
    _fields_ = [
        ("back", C.c_void_p),
        ("slot_of", C.c_void_p),
        ("n_tok", C.c_int32),
        ("hidden", C.c_int32),
        ("world", C.c_int32),
        ("y", C.c_void_p),
        ("y_row_stride", C.c_int64),
    ]


class CacheStats(C.Structure):
    """nvmoe_cache_stats (the device buffer is an int64 tensor of the same layout)."""
    _fields_ = [(n, C.c_int64) for n in (
        "calls", "decode_calls", "gpu_hits", "gpu_misses", "decode_gpu_hits",
        "decode_gpu_misses", "refill_bytes", "error_calls")]


class PruneArgs(C.Structure):
    """nvmoe_prune_args."""
    _fields_ = [
        ("ids", C.c_void_p),
        ("ids_row_stride", C.c_int64),
        ("weights", C.c_void_p),
        ("weights_row_stride", C.c_int64),
        ("n_tok", C.c_int32),
        ("top_k", C.c_int32),
        ("slot_of_real", C.c_void_p),
        ("host_slot_of_real", C.c_void_p),
        ("real_in_slot", C.c_void_p),
        ("cache_size", C.c_int32),
        ("n_expert", C.c_int32),
        ("nvme_thresh", C.c_float),
        ("host_thresh", C.c_float),
        ("min_mass", C.c_float),
        ("min_keep", C.c_int32),
        ("is_decode", C.c_int32),
        ("pruned", C.c_void_p),
    ]


class RouterGateArgs(C.Structure):
    _fields_ = [
        ("resid", C.c_void_p),
        ("resid_row_stride", C.c_int64),
        ("delta", C.c_void_p),
        ("delta_row_stride", C.c_int64),
        ("resid_out", C.c_void_p),
        ("resid_out_row_stride", C.c_int64),
        ("norm_weight", C.c_void_p),
        ("eps", C.c_float),
        ("x_out", C.c_void_p),
        ("x_out_row_stride", C.c_int64),
        ("gate_weight", C.c_void_p),
        ("gate_row_stride", C.c_int64),
        ("logit_bias", C.c_void_p),
        ("logits", C.c_void_p),
        ("logits_row_stride", C.c_int64),
        ("n_tok", C.c_int32),
        ("hidden", C.c_int32),
        ("n_expert", C.c_int32),
        ("top_k", C.c_int32),
        ("router_mode", C.c_int32),
        ("router_bias", C.c_void_p),
        ("norm_topk", C.c_int32),
        ("routed_scaling", C.c_float),
        ("out_ids", C.c_void_p),
        ("out_weights", C.c_void_p),
        ("tickets", C.c_void_p),
    ]


# name -> (restype, argtypes); must match include/nvmoe_b200.h
SIGNATURES = {
    "nvmoe_last_error": (C.c_char_p, []),
    "nvmoe_version": (C.c_char_p, []),
    "nvmoe_router_topk": (C.c_int, [C.c_void_p, C.c_int64, C.c_int, C.c_int, C.c_int, C.c_int,
                                    C.c_void_p, C.c_int, C.c_float, C.c_void_p, C.c_int64,
                                    C.c_void_p, C.c_int64, C.c_void_p]),
    "nvmoe_remap": (C.c_int, [C.POINTER(SlotTable), C.c_void_p, C.c_int64, C.c_int, C.c_int,
                              C.c_int, C.c_void_p, C.c_int64, C.POINTER(MissList), C.c_void_p]),
    "nvmoe_dequant_nvfp4": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int64, C.c_int64,
                                      C.c_void_p, C.c_void_p]),
    "nvmoe_dequant_q2_k": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "nvmoe_dequant_iq2_xxs": (C.c_int, [C.c_void_p, C.c_int64, C.c_void_p, C.c_void_p]),
    "nvmoe_set_iq2xxs_grid": (C.c_int, [C.c_void_p]),
    "nvmoe_moe_ffn_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int, C.c_int]),
    "nvmoe_moe_ffn": (C.c_int, [C.POINTER(FfnArgs), C.c_void_p]),
    "nvmoe_moe_ffn_prepare": (C.c_int, [C.POINTER(FfnArgs), C.c_void_p]),
    "nvmoe_moe_ffn_execute": (C.c_int, [C.POINTER(FfnArgs), C.c_void_p]),
    "nvmoe_moe_ffn_path": (C.c_int, [C.POINTER(FfnArgs)]),
    "nvmoe_moe_ffn_noalloc": (C.c_int, [C.POINTER(FfnArgs), C.c_void_p]),
    "nvmoe_moe_ffn_prefill_workspace_size": (C.c_size_t, [C.c_int, C.c_int, C.c_int, C.c_int,
                                                          C.c_int]),
    "nvmoe_moe_ffn_prefill": (C.c_int, [C.POINTER(FfnArgs), C.c_void_p]),
    "nvmoe_slru_create": (C.c_void_p, [C.c_double]),
    "nvmoe_slru_destroy": (None, [C.c_void_p]),
    "nvmoe_slru_set_capacity_hint": (None, [C.c_void_p, C.c_int64]),
    "nvmoe_slru_insert_new": (None, [C.c_void_p, C.c_int64]),
    "nvmoe_slru_touch": (None, [C.c_void_p, C.c_int64]),
    "nvmoe_slru_contains": (C.c_int, [C.c_void_p, C.c_int64]),
    "nvmoe_slru_size": (C.c_int64, [C.c_void_p]),
    "nvmoe_slru_pop_lru": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64)]),
    "nvmoe_slru_pop_lru_excluding": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64), C.c_int,
                                               C.POINTER(C.c_int64)]),
    "nvmoe_slru_discard": (None, [C.c_void_p, C.c_int64]),
    "nvmoe_host_tier_create": (C.c_void_p, [C.c_int32, C.c_int32, C.c_double]),
    "nvmoe_host_tier_destroy": (None, [C.c_void_p]),
    "nvmoe_host_tier_resolve": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                          C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "nvmoe_host_tier_tables": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p]),
    "nvmoe_host_tier_stats": (C.c_int, [C.c_void_p, C.POINTER(C.c_int64),
                                        C.POINTER(C.c_int64)]),
    "nvmoe_cache_stats_add": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int64,
                                        C.c_void_p]),
    "nvmoe_prune_tail": (C.c_int, [C.POINTER(PruneArgs), C.c_void_p]),
    "nvmoe_refill_async": (C.c_int, [C.POINTER(RefillBank), C.c_int, C.c_void_p, C.c_void_p,
                                     C.c_int, C.c_int32, C.c_int32, C.c_void_p, C.c_void_p,
                                     C.c_void_p]),
    "nvmoe_refill_gather": (C.c_int, [C.POINTER(RefillBank), C.c_int, C.POINTER(MissList),
                                      C.c_void_p, C.c_int32, C.c_void_p]),
    "nvmoe_decode_layer": (C.c_int, [C.POINTER(DecodeArgs), C.c_void_p]),
    "nvmoe_router_gate": (C.c_int, [C.POINTER(RouterGateArgs), C.c_void_p]),
    "nvmoe_ep_row_bytes": (C.c_size_t, [C.c_int, C.c_int]),
    "nvmoe_ep_dispatch": (C.c_int, [C.POINTER(EpDispatchArgs), C.c_void_p]),
    "nvmoe_ep_combine": (C.c_int, [C.POINTER(EpCombineArgs), C.c_void_p]),
    "nvmoe_probe_fp4_mma": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p]),
}

_lock = threading.Lock()
_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """The loaded library (raises if it is missing: the CUDA path has no fallback)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise RuntimeError(
                    f"{LIB_PATH.name} is not built; run `python -m nvmoe_b200.build` "
                    "(the CUDA extension is required, there is no CPU fallback)")
            handle = C.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(handle, name)
                fn.restype = res
                fn.argtypes = args
            _lib = handle
    return _lib


def check(status: int, where: str) -> None:
    if status != NVMOE_OK:
        detail = ""
        if status == NVMOE_ERR_CUDA:
            detail = (lib().nvmoe_last_error() or b"").decode(errors="replace")
        raise NvmoeError(status, where, detail)
