"""Build recipe for the in-tree CUDA library ``lmpool_b200/_kvx.so``.

The library is compiled with nvcc for sm_100a only (B200) and links the CUDA
runtime statically, so it needs nothing from PyTorch and loads on a machine
without a GPU (driver entry points are resolved at first use). Python reaches
it through ctypes (``lmpool_b200/_capi.py``); the C ABI is ``include/kvx.h``.

Usage: ``python -m lmpool_b200._build [--verbose]``.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO_ROOT = PKG_DIR.parent
SOURCES = [PKG_DIR / "csrc" / "kvx.cu"]
HEADERS = [REPO_ROOT / "include" / "kvx.h", PKG_DIR / "csrc" / "kvx_device.cuh"]
OUTPUT = PKG_DIR / "_kvx.so"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-lineinfo",
    "-shared",
    "-Xcompiler",
    "-fPIC,-O2",
    "-cudart",
    "static",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the KV data path needs the CUDA 12.9 toolchain to build")


def is_stale() -> bool:
    if not OUTPUT.exists():
        return True
    out_m = OUTPUT.stat().st_mtime
    return any(p.stat().st_mtime > out_m for p in SOURCES + HEADERS)


def build(force: bool = False, verbose: bool = False, ptxas_info: bool = False) -> Path:
    """Compile the library if a source is newer than the built file."""
    if not force and not is_stale():
        return OUTPUT
    tmp = OUTPUT.with_suffix(".so.tmp")
    cmd = [nvcc_path(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", str(REPO_ROOT / "include"), "-I", str(PKG_DIR / "csrc")]
    if ptxas_info:
        cmd += ["-Xptxas", "-v"]
    cmd += ["-o", str(tmp), *map(str, SOURCES)]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose or ptxas_info:
        sys.stderr.write(res.stdout + res.stderr)
    os.replace(tmp, OUTPUT)
    return OUTPUT


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print registers/spills per kernel")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose, ptxas_info=args.ptxas_info))


if __name__ == "__main__":
    main()
