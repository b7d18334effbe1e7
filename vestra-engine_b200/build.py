"""Builds libvestra_attn.so (all CUDA sources, sm_100a) into vestra-engine_b200/_build/.

Usage: python vestra-engine_b200/build.py [--verbose-ptxas] [--force]

The library is a plain shared object with a C ABI (include/vestra_attn.h); it
statically links the CUDA runtime and needs nothing from PyTorch.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(BUILD, "libvestra_attn.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
              "--expt-relaxed-constexpr", "-I" + os.path.join(ROOT, "include")]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _host_compiler_flags() -> list[str]:
    # The image exports CXX=/opt/gcc/bin/g++ (a wrapper); nvcc finds the system g++ itself.
    gxx = "/usr/bin/g++"
    return ["-ccbin", gxx] if os.path.exists(gxx) else []


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(verbose_ptxas: bool = False, force: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    headers = glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) + \
        glob.glob(os.path.join(ROOT, "include", "*.h"))
    objs = []
    jobs = []
    for src in sources():
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or verbose_ptxas or _stale(obj, [src] + headers):
            cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *_host_compiler_flags(), "-c", src, "-o", obj]
            if verbose_ptxas:
                cmd += ["-Xptxas", "-v"]
            jobs.append(cmd)
    with cf.ThreadPoolExecutor(max_workers=min(8, max(1, len(jobs)))) as ex:
        for cmd, res in zip(jobs, ex.map(lambda c: subprocess.run(c, capture_output=True, text=True), jobs)):
            if res.returncode != 0:
                sys.stderr.write(res.stdout + res.stderr)
                raise RuntimeError("nvcc failed: " + " ".join(cmd))
            if verbose_ptxas:
                sys.stderr.write(res.stderr)
    if force or jobs or _stale(LIB, objs):
        cmd = [nvcc(), *ARCH, *_host_compiler_flags(), "-shared", "-o", LIB, *objs, "-lcudart_static",
               "-ldl", "-lpthread", "-lrt"]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            sys.stderr.write(res.stdout + res.stderr)
            raise RuntimeError("link failed: " + " ".join(cmd))
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(verbose_ptxas=a.verbose_ptxas, force=a.force))
