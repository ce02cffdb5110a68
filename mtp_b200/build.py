"""Build libmtp_b200.so in-tree with nvcc for sm_100a.

The library is plain C ABI (no torch types), compiled directly by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` and the CUDA runtime linked
statically, so it loads the same way from ctypes, a cgo stub or any other FFI.

    python -m mtp_b200.build          # build if sources changed
    python -m mtp_b200.build --force  # rebuild
"""
from __future__ import annotations

import argparse
import hashlib
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
LIBDIR = PKG / "lib"
LIB = LIBDIR / "libmtp_b200.so"
STAMP = LIBDIR / "libmtp_b200.stamp"

SOURCES = ["capi.cu", "router_align.cu", "gptq.cu", "moe_fused.cu", "moe_prefill.cu", "predictor.cu", "prefetch.cu",
           "noalloc.cu"]
HEADERS = ["common.cuh", "internal.cuh", "route.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or "/usr/local/cuda/bin/nvcc"
    return cand if Path(cand).exists() else "nvcc"


def _digest(extra: list[str]) -> str:
    h = hashlib.sha256()
    for f in sorted(SOURCES + HEADERS):
        h.update((CSRC / f).read_bytes())
    h.update((INCLUDE / "mtp_b200.h").read_bytes())
    h.update(" ".join(extra).encode())
    return h.hexdigest()


def flags(verbose_ptxas: bool = False) -> list[str]:
    f = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden", "-I", str(INCLUDE), "-I", str(CSRC), *ARCH]
    if verbose_ptxas:
        f += ["-Xptxas", "-v"]
    return f


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> Path:
    LIBDIR.mkdir(parents=True, exist_ok=True)
    fl = flags(verbose_ptxas)
    digest = _digest(fl)
    if not force and LIB.exists() and STAMP.exists() and STAMP.read_text().strip() == digest:
        return LIB
    objs = []
    for src in SOURCES:
        obj = LIBDIR / (Path(src).stem + ".o")
        cmd = [nvcc(), *fl, "-c", str(CSRC / src), "-o", str(obj)]
        if not quiet:
            print(" ".join(cmd), flush=True)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *objs]
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    for o in objs:
        Path(o).unlink(missing_ok=True)
    STAMP.write_text(digest)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--ptxas-verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.ptxas_verbose))
    sys.exit(0)
