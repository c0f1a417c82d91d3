"""Build libminitp_b200.so (the sm_100a kernels behind the C ABI) in-tree.

    python -m minitp_b200.build [--force] [--verbose]

The library is compiled by nvcc for sm_100a only and written to
``minitp_b200/_lib/libminitp_b200.so``. Nothing is compiled at import time;
``minitp_b200._lib`` raises if the library is missing.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(REPO, "include")
OUT_DIR = os.path.join(PKG, "_lib")
LIB_PATH = os.path.join(OUT_DIR, "libminitp_b200.so")

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr"]
MAIN_SOURCE = os.path.join(CSRC, "capi.cu")


def _inputs() -> list[str]:
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(INCLUDE, "minitp_b200.h"))
    return files


def needs_build() -> bool:
    if not os.path.exists(LIB_PATH):
        return True
    t = os.path.getmtime(LIB_PATH)
    return any(os.path.getmtime(f) > t for f in _inputs())


def nvcc() -> str:
    exe = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(exe):
        raise RuntimeError("nvcc not found: the CUDA toolkit is required to build minitp_b200")
    return exe


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile the library if any source is newer than it; returns its path."""
    if not force and not needs_build():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB_PATH + ".tmp"
    cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-I", INCLUDE, "-o", tmp, MAIN_SOURCE]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
        print(" ".join(cmd), flush=True)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stderr[-8000:]}")
    if verbose:
        print(res.stderr, flush=True)
    os.replace(tmp, LIB_PATH)
    return LIB_PATH


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
