"""Build ``needle_b200/_lib/libneedle_b200.so`` from ``needle_b200/csrc`` with nvcc
(and the small host-side CPython extension ``_steppack`` with gcc).

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


HOST_SRC = os.path.join(PKG, "host", "steppack.c")


def host_ext_path() -> str:
    import sysconfig
    return os.path.join(OUT_DIR, "_steppack" + sysconfig.get_config_var("EXT_SUFFIX"))


def build_host(force: bool = False, verbose: bool = False) -> str:
    """The CPython extension with the host-side step packing (gcc, -O2)."""
    import sysconfig
    out = host_ext_path()
    stamp = out + ".srchash"
    with open(HOST_SRC, "rb") as fh:
        digest = hashlib.sha256(fh.read() + sys.version.encode()).hexdigest()
    if not force and os.path.exists(out) and os.path.exists(stamp):
        with open(stamp) as fh:
            if fh.read().strip() == digest:
                return out
    os.makedirs(OUT_DIR, exist_ok=True)
    cc = os.environ.get("CC") or shutil.which("gcc") or "cc"
    cmd = [cc, "-O2", "-fPIC", "-shared", "-Wall", "-I", sysconfig.get_paths()["include"],
           HOST_SRC, "-o", out + ".tmp"]
    if verbose:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(out + ".tmp", out)
    with open(stamp, "w") as fh:
        fh.write(digest)
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.ptxas_v else []
    print(build(force=a.force or a.ptxas_v, verbose=True, extra=extra))
    print(build_host(force=a.force, verbose=True))


if __name__ == "__main__":
    sys.exit(main())
