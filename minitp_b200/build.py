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
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr"]
# translation units, compiled in parallel: the C ABI with the kernel chain, and
# the decode megakernel's bf16 and fp32 instantiations
SOURCES = [os.path.join(CSRC, f) for f in ("capi.cu", "decode_mk_bf16.cu", "decode_mk_f32.cu")]
OBJ_DIR = os.path.join(REPO, "_build")


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


def build(force: bool = False, verbose: bool = False, defines: tuple = (), out: str | None = None) -> str:
    """Compile the library if any source is newer than it; returns its path.

    `defines` (e.g. ``("MTPB_DECODE_TRACE=1",)``, the decode megakernel's phase
    trace) and `out` build a variant elsewhere; such a build always compiles.
    """
    lib_path = out or LIB_PATH
    if not force and not defines and out is None and not needs_build():
        return LIB_PATH
    os.makedirs(OUT_DIR, exist_ok=True)
    os.makedirs(OBJ_DIR, exist_ok=True)
    objs, procs = [], []
    for src in SOURCES:
        obj = os.path.join(OBJ_DIR, os.path.basename(src).replace(".cu", f".{os.getpid()}.o"))
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, *(f"-D{d}" for d in defines), "-I", INCLUDE, "-c", "-o", obj, src]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), flush=True)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True)))
        objs.append(obj)
    errors = []
    for src, pr in procs:
        out, err = pr.communicate()
        if pr.returncode != 0:
            errors.append(f"nvcc failed on {os.path.basename(src)} ({pr.returncode}):\n{err[-8000:]}")
        elif verbose:
            print(err, flush=True)
    try:
        if errors:
            raise RuntimeError("\n".join(errors))
        tmp = lib_path + f".{os.getpid()}.tmp"
        link = [nvcc(), *ARCH_FLAGS, "-shared", "-o", tmp, *objs]
        res = subprocess.run(link, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed ({res.returncode}):\n{res.stderr[-8000:]}")
        os.replace(tmp, lib_path)
    finally:
        for o in objs:
            if os.path.exists(o):
                os.remove(o)
    return lib_path


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose=a.verbose))


if __name__ == "__main__":
    main()
