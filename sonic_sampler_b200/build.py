"""Build the in-tree CUDA library `sonic_sampler_b200/_lib/libsonic_b200.so` for sm_100a.

    python -m sonic_sampler_b200.build [--force]

nvcc cross-compiles without a GPU. The library links the CUDA runtime statically, so it
only needs the driver at run time.
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PACKAGE_DIR = Path(__file__).resolve().parent
CSRC = PACKAGE_DIR / "csrc"
OUT = PACKAGE_DIR / "_lib" / "libsonic_b200.so"
# diagnostic variant with per-phase timing stamps (python -m sonic_sampler_b200.phases)
STAMPS_OUT = PACKAGE_DIR / "_lib" / "libsonic_b200_stamps.so"
SOURCES = [CSRC / "sampler.cu"]
HEADERS = [CSRC / "common.cuh", CSRC / "exports.map", PACKAGE_DIR.parent / "include" / "sonic_b200.h"]

NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    # exact bf16/fp32 reproduction: no implicit multiply-add contraction
    "--fmad=false",
    "-Xcompiler", "-fPIC", "-shared",
    "-cudart", "static",
    "-Xlinker", f"--version-script={CSRC / 'exports.map'}",
]


def nvcc_path() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cand.is_file():
        return str(cand)
    raise RuntimeError("nvcc not found (set CUDA_HOME or put nvcc on PATH)")


def stale(out: Path = OUT) -> bool:
    if not out.is_file():
        return True
    t = out.stat().st_mtime
    return any(p.stat().st_mtime > t for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, stamps: bool = False) -> Path:
    """Build the product library, or with `stamps` the phase-stamp diagnostic variant."""
    out = STAMPS_OUT if stamps else OUT
    if not force and not stale(out):
        return out
    out.parent.mkdir(parents=True, exist_ok=True)
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *NVCC_FLAGS, *(["-DSONIC_PHASE_STAMPS"] if stamps else []), "-o", str(tmp),
           *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, stamps="--stamps" in sys.argv))
