"""Builds ``libaethermoe.so`` (the C-ABI library) in-tree for sm_100a.

Every ``csrc/*.cu`` is compiled by nvcc with
``-gencode arch=compute_100a,code=sm_100a`` into ``_build/`` and linked into
``aethermoe_b200/libaethermoe.so`` (CUDA runtime linked statically; NCCL
dynamically).  Usage: ``python -m aethermoe_b200.build [-v] [--force]``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(ROOT, "_build")
LIB = os.path.join(HERE, "libaethermoe.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall",
         "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]
# Per-file extra flags (none at present).
FILE_FLAGS: dict = {}


def _nvcc():
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build aethermoe_b200")


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".h", ".cuh"))]
    hs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE) if f.endswith(".h")]
    return hs


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}")
    if verbose and r.stdout.strip():
        print(r.stdout, flush=True)
    return r.stdout


def build(verbose=False, force=False, ptxas_info=False):
    """Compiles the library if any source changed; returns the .so path."""
    nvcc = _nvcc()
    os.makedirs(BUILD, exist_ok=True)
    headers = _headers()
    objs, jobs = [], []
    for src in _sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, [src, os.path.abspath(__file__)] + headers):
            cmd = [nvcc] + ARCH + FLAGS + FILE_FLAGS.get(os.path.basename(src), []) + \
                (["-Xptxas", "-v"] if ptxas_info else []) + ["-c", src, "-o", obj]
            jobs.append(cmd)
    out = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, len(jobs))) as ex:
            for o in ex.map(lambda c: _run(c, verbose), jobs):
                out.append(o)
    if force or jobs or _stale(LIB, objs):
        _run([nvcc] + ARCH + ["-shared", "-o", LIB] + objs + ["-ldl", "-lpthread"], verbose)
    if ptxas_info:
        print("\n".join(out))
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="--force" in sys.argv,
          ptxas_info="--ptxas" in sys.argv)
    print(LIB)
