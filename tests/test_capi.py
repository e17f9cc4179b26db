"""The C-ABI library loads and exports every entry point include/nvmoe_b200.h declares (CPU)."""
import ctypes
import re
from pathlib import Path

from nvmoe_b200 import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "nvmoe_b200.h"


def declared_functions() -> set[str]:
    text = HEADER.read_text()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(r"\b(nvmoe_[a-z0-9_]+)\s*\(", text))


def test_library_loads_and_reports_version():
    lib = _lib.lib()
    assert lib.nvmoe_version().decode().startswith("nvmoe_b200")


def test_every_declared_symbol_is_exported_and_bound():
    lib = _lib.lib()
    names = declared_functions()
    assert len(names) >= 20
    for n in sorted(names):
        assert hasattr(lib, n), f"{n} declared in the header but not exported"
        assert n in _lib.SIGNATURES, f"{n} has no ctypes signature in nvmoe_b200/_lib.py"


def test_struct_sizes_match_c_layout():
    # 8 pointers/int64 + 4 int32 etc.: the ctypes mirrors must have the C sizes
    assert ctypes.sizeof(_lib.SlotTable) == 4 * 8 + 4 * 4
    assert ctypes.sizeof(_lib.MissList) == 7 * 8 + 8
    assert ctypes.sizeof(_lib.MatrixBank) == 8 * 8
    assert ctypes.sizeof(_lib.ExpertPool) == 16 + 3 * 64
    assert ctypes.sizeof(_lib.RefillBank) == 5 * 8


def test_host_side_argument_validation_without_gpu():
    lib = _lib.lib()
    # null / invalid arguments are rejected before any CUDA call
    assert lib.nvmoe_router_topk(None, 0, 1, 0, 1, 0, None, 1, 1.0, None, 1, None, 1, None) == \
        _lib.NVMOE_ERR_INVALID_ARG
    assert lib.nvmoe_remap(None, None, 0, 1, 1, 1, None, 0, None, None) == _lib.NVMOE_ERR_INVALID_ARG
    assert lib.nvmoe_moe_ffn(None, None) == _lib.NVMOE_ERR_INVALID_ARG
    assert lib.nvmoe_moe_ffn_workspace_size(8, 10, 2048, 512, 128) > 0
    assert lib.nvmoe_moe_ffn_workspace_size(0, 10, 2048, 512, 128) == 0


def test_struct_layouts_match_a_c_compiler(tmp_path):
    """Every ctypes mirror has the size and field offsets gcc gives the header's structs."""
    import shutil
    import subprocess

    import pytest
    gcc = shutil.which("gcc")
    if gcc is None:
        pytest.skip("gcc not available")
    mirrors = {"nvmoe_slot_table": _lib.SlotTable, "nvmoe_miss_list": _lib.MissList,
               "nvmoe_matrix_bank": _lib.MatrixBank, "nvmoe_expert_pool": _lib.ExpertPool,
               "nvmoe_ffn_args": _lib.FfnArgs, "nvmoe_refill_bank": _lib.RefillBank,
               "nvmoe_decode_args": _lib.DecodeArgs,
               "nvmoe_router_gate_args": _lib.RouterGateArgs,
               "nvmoe_ep_dispatch_args": _lib.EpDispatchArgs,
               "nvmoe_ep_combine_args": _lib.EpCombineArgs,
               "nvmoe_cache_stats": _lib.CacheStats, "nvmoe_prune_args": _lib.PruneArgs}
    lines = ['#include <stdio.h>', '#include <stddef.h>', '#include "nvmoe_b200.h"',
             'int main(void) {']
    for cname, py in mirrors.items():
        lines.append(f'printf("{cname} size %zu\\n", sizeof({cname}));')
        for fname, _ in py._fields_:
            lines.append(f'printf("{cname} {fname} %zu\\n", offsetof({cname}, {fname}));')
    lines += ["return 0;", "}"]
    src = tmp_path / "layout.c"
    src.write_text("\n".join(lines))
    exe = tmp_path / "layout"
    subprocess.run([gcc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], check=True, capture_output=True, text=True).stdout
    got = {}
    for ln in out.splitlines():
        c, f, v = ln.split()
        got[(c, f)] = int(v)
    for cname, py in mirrors.items():
        assert got[(cname, "size")] == ctypes.sizeof(py), cname
        for fname, _ in py._fields_:
            assert got[(cname, fname)] == getattr(py, fname).offset, (cname, fname)
