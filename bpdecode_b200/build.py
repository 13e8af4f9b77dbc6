"""Compile the sm_100a CUDA library in-tree: ``libbpdecode_b200.so`` beside
this file (the C ABI declared in ``include/bpdecode_b200.h``).

    python -m bpdecode_b200.build [--verbose]

Each ``csrc/*.cu`` is compiled to an object in parallel with
``nvcc -gencode arch=compute_100a,code=sm_100a -lineinfo -O3`` and linked
into one shared library with the CUDA runtime linked statically, so the
library needs no CUDA toolkit on the machine that loads it.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbpdecode_b200.so")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = "/usr/local/cuda/bin/nvcc"
    if os.path.exists(cand):
        return cand
    raise RuntimeError("nvcc not found")


def _flags(verbose: bool) -> list[str]:
    f = [*ARCH, "-lineinfo", "-O3", "-std=c++17", "-Xcompiler", "-fPIC",
         "-I", os.path.join(ROOT, "include"), "--expt-relaxed-constexpr"]
    if verbose:
        f += ["-Xptxas", "-v"]
    return f


def _compile(src: str, verbose: bool) -> tuple[str, str]:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if (not verbose and os.path.exists(obj)
            and os.path.getmtime(obj) >= max(os.path.getmtime(p) for p in _deps(src))):
        return obj, ""
    cmd = [nvcc(), *_flags(verbose), "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, r.stderr


def _deps(src: str) -> list[str]:
    return [src, *glob.glob(os.path.join(CSRC, "*.cuh")),
            os.path.join(ROOT, "include", "bpdecode_b200.h")]


def build(verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, verbose), srcs))
    objs = [o for o, _ in results]
    if verbose:
        for _, log in results:
            if log:
                print(log)
    if (not os.path.exists(LIB)
            or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs)):
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true", help="print -Xptxas -v resource usage")
    print(build(ap.parse_args().verbose))
