"""Build libcozy_ulysses.so in-tree with nvcc for sm_100a.

The library has no Python or torch types in its interface (include/cozy_ulysses.h); the Python
host side loads it with ctypes (`cozy_runtime_b200._lib`). Run `python -m cozy_runtime_b200.build`
or call `build()`; `__graft_entry__.build()` does.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE = Path(__file__).resolve().parent
ROOT = PACKAGE.parent
CSRC = PACKAGE / "csrc"
LIBRARY = PACKAGE / "libcozy_ulysses.so"
SOURCES = [
    "attention_fwd.cu", "stage.cu", "fp8.cu", "peer.cu", "layer.cu", "noalloc.cu", "narrow.cu", "capi.cu",
]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
#: Sources compiled with IEEE fp32 semantics (denormals kept, exact division and square root):
#: the int8 wire's law must round as the reference's CPU arithmetic does.
EXACT = {"narrow.cu"}


def nvcc() -> str:
    found = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(found).exists():
        raise RuntimeError("nvcc not found: the CUDA toolkit is needed to build the library")
    return found


def flags(verbose: bool = False, exact: bool = False) -> list[str]:
    out = [
        *ARCH,
        "-O3",
        "-std=c++17",
        "-lineinfo",
        *(["-ftz=false", "-prec-div=true", "-prec-sqrt=true"] if exact else ["--use_fast_math"]),
        "-Xcompiler",
        "-fPIC,-fvisibility=hidden",
        "-I",
        str(ROOT / "include"),
    ]
    if verbose:
        out += ["-Xptxas", "-v"]
    return out


def stale() -> bool:
    if not LIBRARY.exists():
        return True
    built = LIBRARY.stat().st_mtime
    inputs = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return any(p.stat().st_mtime > built for p in inputs)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not stale():
        return LIBRARY
    out_dir = PACKAGE / "_build"
    out_dir.mkdir(exist_ok=True)
    objects = []
    for source in SOURCES:
        obj = out_dir / (Path(source).stem + ".o")
        cmd = [nvcc(), *flags(verbose, source in EXACT), "-c", str(CSRC / source), "-o", str(obj)]
        subprocess.run(cmd, check=True)
        objects.append(str(obj))
    tmp = LIBRARY.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objects]
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIBRARY)
    return LIBRARY


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(LIBRARY)
