"""nvmoe_b200 — B200-native routed-expert FFN over a VRAM expert-slot cache.

The CUDA kernels and the C ABI live in libnvmoe_b200.so (built in-tree by
``python -m nvmoe_b200.build``); this package is the host side: ctypes bindings, torch-facing
ops, the offload-cache hook (`SlotCache`) and synthetic data generators.
"""
__version__ = "0.1.0"

from . import formats, synth  # noqa: F401
