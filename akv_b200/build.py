"""Build ``libakv_b200.so`` (the C ABI of include/akv_b200.h) for sm_100a.

    python -m akv_b200.build [--force] [--verbose]

Compiles every ``csrc/*.cu`` with nvcc for ``sm_100a`` only and links them
into ``akv_b200/libakv_b200.so`` in the source tree, so the built library
travels with the tree.  ``-Xptxas -v`` output (registers, spills, shared
memory) is written to ``akv_b200/_build/ptxas.txt``.
"""

from __future__ import annotations

import os
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libakv_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xptxas", "-v",
         "--expt-relaxed-constexpr"]


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    headers.append(os.path.join(INCLUDE, "akv_b200.h"))
    objects, logs = [], []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objects.append(obj)
        if force or _stale(obj, [src] + headers):
            cmd = [NVCC, *ARCH, *FLAGS, "-I", INCLUDE, "-I", CSRC, "-c", src, "-o", obj]
            res = subprocess.run(cmd, capture_output=True, text=True)
            logs.append(f"== {os.path.basename(src)}\n{res.stderr}")
            if res.returncode != 0:
                sys.stderr.write(res.stderr)
                raise RuntimeError(f"nvcc failed on {src}")
            if verbose:
                sys.stderr.write(res.stderr)
    if logs:
        with open(os.path.join(BUILD, "ptxas.txt"), "w") as f:
            f.write("\n".join(logs))
    if force or _stale(LIB, objects):
        cmd = [NVCC, *ARCH, "-shared", "-o", LIB, *objects, "-lcudart"]
        subprocess.run(cmd, check=True)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="--verbose" in sys.argv))
