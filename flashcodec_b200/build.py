"""Build libflashcodec_sm100.so in-tree with nvcc (sm_100a only).

    python -m flashcodec_b200.build [--force]

The library is a plain C-ABI shared object (include/flashcodec_b200.h); it
links the CUDA runtime statically and has no dependency on PyTorch.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "libflashcodec_sm100.so"
SOURCES = sorted(CSRC.glob("*.cu"))
HEADERS = sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "flashcodec_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden",
    "-Xptxas", "-warn-spills",
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the flashcodec_b200 CUDA library cannot be built")


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False) -> Path:
    """Compile every .cu under csrc/ into libflashcodec_sm100.so (in-tree)."""
    if not force and up_to_date():
        return LIB
    out = PKG / "_build"
    out.mkdir(exist_ok=True)
    objs = []
    newest_header = max(p.stat().st_mtime for p in HEADERS)
    for src in SOURCES:
        obj = out / (src.stem + ".o")
        fresh = (not force and obj.exists() and
                 obj.stat().st_mtime >= max(src.stat().st_mtime, newest_header))
        if not fresh:
            cmd = [nvcc(), *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
            if verbose:
                print(" ".join(cmd), flush=True)
            subprocess.check_call(cmd)
        objs.append(str(obj))
    tmp = LIB.with_suffix(f".{os.getpid()}.tmp")
    subprocess.check_call([nvcc(), "-gencode", "arch=compute_100a,code=sm_100a", "-shared",
                           "-o", str(tmp), *objs])
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
