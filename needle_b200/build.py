"""Build ``needle_b200/_lib/libneedle_b200.so`` from ``needle_b200/csrc`` with nvcc.

The library is a plain shared object with a C ABI (``include/needle_b200.h``);
it does not link against torch.  It is compiled for sm_100a only and built
in-tree so that the file travels with the repository snapshot.

    python -m needle_b200.build            # build if sources changed
    python -m needle_b200.build --force    # always rebuild
"""
from __future__ import annotations

import argparse
import hashlib
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
OUT_DIR = os.path.join(PKG, "_lib")
LIB = os.path.join(OUT_DIR, "libneedle_b200.so")
STAMP = LIB + ".srchash"


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    files = [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))]
    files.append(os.path.join(ROOT, "include", "needle_b200.h"))
    return files


def _hash(flags) -> str:
    h = hashlib.sha256(" ".join(flags).encode())
    for f in _sources():
        with open(f, "rb") as fh:
            h.update(fh.read())
    return h.hexdigest()


def flags(extra=()):
    return [
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17",
        "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
        "--expt-relaxed-constexpr",
        "-shared",
        *extra,
    ]


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    f = flags(extra)
    digest = _hash(f)
    if not force and os.path.exists(LIB) and os.path.exists(STAMP):
        with open(STAMP) as fh:
            if fh.read().strip() == digest:
                return LIB
    os.makedirs(OUT_DIR, exist_ok=True)
    tmp = LIB + ".tmp"
    cmd = [_nvcc(), *f, os.path.join(CSRC, "needle_b200.cu"), "-o", tmp]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    with open(STAMP, "w") as fh:
        fh.write(digest)
    return LIB


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=True, extra=extra))


if __name__ == "__main__":
    sys.exit(main())
