"""Build libsca2b200.so in-tree with nvcc for sm_100a (no JIT cache, no torch extension).

    python -m sca2_b200.build          # rebuild if any source is newer than the library
    python -m sca2_b200.build --force

The library is a plain C-ABI shared object (include/sca2b200.h); the Python host side
binds it with ctypes.
"""
from __future__ import annotations

import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
LIB = os.path.join(PKG, "libsca2b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
         "-Xcompiler", "-fvisibility=hidden"]


def _nvcc():
    for c in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if c and os.path.exists(c):
            return c
    raise RuntimeError("nvcc not found: the sca2b200 CUDA library cannot be built")


def sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h")))


def up_to_date(lib=LIB):
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(s) <= t for s in sources() + headers() + [__file__])


def build(force=False, verbose=False, lib=LIB, extra=()):
    """Compile every .cu under csrc/ into one shared library (separate objects, one link)."""
    if not force and up_to_date(lib):
        return lib
    nvcc = _nvcc()
    objdir = os.path.join(PKG, "_build")
    os.makedirs(objdir, exist_ok=True)
    objs = []
    procs = []
    for src in sources():
        obj = os.path.join(objdir, os.path.basename(src) + ".o")
        cmd = [nvcc, *ARCH, *FLAGS, *extra, "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(obj)
    failed = []
    for src, p in procs:
        out = p.communicate()[0].decode(errors="replace")
        if p.returncode != 0:
            failed.append(f"{src}:\n{out}")
        elif verbose and out.strip():
            print(out)
    if failed:
        raise RuntimeError("nvcc failed:\n" + "\n".join(failed))
    tmp = lib + ".tmp"
    cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart"]
    if verbose:
        print(" ".join(cmd))
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n" + r.stdout.decode(errors="replace"))
    os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print("built", LIB)
