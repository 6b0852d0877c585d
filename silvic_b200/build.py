"""Builds the B200 backend: every CUDA source of silvic_b200/csrc into silvic_b200/_lib/libsilvic_b200.so.

The kernels are compiled for sm_100a only (`-gencode arch=compute_100a,code=sm_100a`), with `--fmad=false` so no
floating-point multiply and add are fused (the split search and the gradients are bit-exact restatements of the
reference's IEEE operations). NCCL comes from the `nvidia-nccl` wheel PyTorch uses, so a process that imports
torch and loads this library shares one NCCL.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
CSRC = PACKAGE / "csrc"
LIB_DIR = PACKAGE / "_lib"
BUILD_DIR = PACKAGE.parent / "_build" / "silvic_b200"
LIBRARY = LIB_DIR / "libsilvic_b200.so"
SOURCES = ["hist.cu", "partition.cu", "split.cu", "grow.cu", "iter.cu", "lambdarank.cu", "binning.cu", "diag.cu", "backend.cu"]
HEADERS = ["common.cuh", "hist.cuh", "hist_device.cuh", "partition.cuh", "search.cuh", "train.cuh", "iter.cuh",
           "fused.cuh", "steps.cuh", "binning.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nccl_dirs() -> tuple[Path, Path]:
    """The include and lib directories of the NCCL wheel next to torch."""
    import importlib.util

    spec = importlib.util.find_spec("nvidia")
    roots = list(spec.submodule_search_locations) if spec and spec.submodule_search_locations else []
    for root in roots:
        base = Path(root) / "nccl"
        if (base / "include" / "nccl.h").exists() and (base / "lib" / "libnccl.so.2").exists():
            return base / "include", base / "lib"
    raise RuntimeError("NCCL headers and library (the nvidia-nccl wheel) not found")


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False) -> Path:
    """Compiles what changed and links the library; returns its path."""
    inc, lib = nccl_dirs()
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + [PACKAGE.parent / "include" / "silvic_b200.h"]
    common = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "--fmad=false", "-Xcompiler", "-fPIC",
              "-Xcompiler", "-Wall", f"-I{inc}"]
    objects = []
    for src in SOURCES:
        obj = BUILD_DIR / (src + ".o")
        objects.append(obj)
        if _stale(obj, [CSRC / src, *headers]):
            cmd = [*common, "-c", str(CSRC / src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), file=sys.stderr)
            subprocess.run(cmd, check=True)
    if _stale(LIBRARY, objects):
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIBRARY), *map(str, objects), f"-L{lib}", "-l:libnccl.so.2",
               f"-Xlinker", f"-rpath={lib}", "-lcudart"]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
    return LIBRARY


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
