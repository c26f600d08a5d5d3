"""Builds the B200 library in-tree: liborbit_wars_cuda.so.

One shared library holds both C ABIs:
  include/orbit_wars_cuda.h  the reference engine's symbols (drop-in)
  include/ow_policy.h        the entity-encoder policy symbols

    python orbit-wars-2d-transformer_b200/build.py [--force]

nvcc cross-compiles for sm_100a (no GPU needed). CUDA runtime is linked
statically; the driver API (tensor-map encoding) is reached through
cudaGetDriverEntryPoint, so no -lcuda is needed at link time.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
LIB_DIR = PKG_DIR / "orbit_wars_b200" / "lib"
LIB = LIB_DIR / "liborbit_wars_cuda.so"
SOURCES = ["ow_policy.cu", "orbit_wars_true2d.cu", "ow_comm.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _deps() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted((REPO / "include").glob("*.h"))


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    t = LIB.stat().st_mtime
    return all(p.stat().st_mtime <= t for p in _deps())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    srcs = [str(CSRC / s) for s in SOURCES if (CSRC / s).exists()]
    cmd = [
        nvcc(), "-std=c++17", "-O3", *ARCH, "-lineinfo", "-shared", "-Xcompiler", "-fPIC",
        "-I", str(REPO / "include"), "-I", str(CSRC),
        "--expt-relaxed-constexpr", *srcs, "-ldl", "-o", str(LIB) + ".tmp",
    ]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB) + ".tmp", LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))
    sys.exit(0)
