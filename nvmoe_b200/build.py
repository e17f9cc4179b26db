"""Builds libnvmoe_b200.so (sm_100a kernels + host C++) in-tree with nvcc.

    python -m nvmoe_b200.build            # incremental
    python -m nvmoe_b200.build --force    # rebuild everything

The library links the CUDA runtime statically, so it carries its own runtime and does not
depend on the version PyTorch ships; stream and device pointers are driver-level handles and
interoperate with PyTorch's.
"""
from __future__ import annotations

import concurrent.futures as cf
import hashlib
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libnvmoe_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-Wall", "--expt-relaxed-constexpr",
                     f"-I{REPO / 'include'}"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _sources() -> list[Path]:
    return sorted([*CSRC.glob("*.cu"), *CSRC.glob("*.cpp")])


def _headers_digest() -> str:
    h = hashlib.sha256()
    for p in sorted([*CSRC.glob("*.cuh"), *CSRC.glob("*.hpp"), *CSRC.glob("*.h"),
                     *(REPO / "include").glob("*.h")]):
        h.update(p.name.encode())
        h.update(p.read_bytes())
    return h.hexdigest()[:16]


def _compile(src: Path, obj: Path) -> None:
    cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    hdr = _headers_digest()
    stamp = BUILD / "headers.digest"
    if stamp.exists() and stamp.read_text() != hdr:
        force = True
    jobs = []
    objs = []
    for src in _sources():
        obj = BUILD / (src.name + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < src.stat().st_mtime:
            jobs.append((src, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            futs = [ex.submit(_compile, s, o) for s, o in jobs]
            for f in futs:
                f.result()
    if jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    stamp.write_text(hdr)
    if verbose:
        print(f"built {LIB} ({len(jobs)} objects compiled)")
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
