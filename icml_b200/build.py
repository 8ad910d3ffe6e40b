"""Build libpgf.so (the C-ABI of include/pgf.h) in-tree with nvcc for sm_100a.

    python -m icml_b200.build            # or: python icml_b200/build.py

Each .cu under icml_b200/csrc is compiled to an object with
``-gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked into
icml_b200/libpgf.so.  Objects are rebuilt only when a source or header is newer.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpgf.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
         "-I" + os.path.join(ROOT, "include")]


def _newest(paths):
    return max((os.path.getmtime(p) for p in paths), default=0.0)


def build(verbose: bool = False, jobs: int = 8) -> str:
    os.makedirs(OBJ, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(ROOT, "include", "*.h"))
    hdr_t = _newest(hdrs)
    procs, objs = [], []
    for src in srcs:
        obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hdr_t):
            continue
        cmd = [NVCC, *ARCH, *FLAGS, "-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd))
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        if len(procs) >= jobs:
            _wait(procs)
            procs = []
    _wait(procs)
    if not os.path.exists(LIB) or os.path.getmtime(LIB) < _newest(objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objs, "-lcuda"]
        if verbose:
            print(" ".join(cmd))
        out = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
        if out.returncode != 0:
            raise RuntimeError("link failed:\n" + out.stdout)
    return LIB


def _wait(procs):
    err = []
    for src, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            err.append(f"{src}:\n{out.decode(errors='replace')}")
        elif out.strip():
            sys.stderr.write(out.decode(errors="replace"))
    if err:
        raise RuntimeError("nvcc failed:\n" + "\n".join(err))


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
