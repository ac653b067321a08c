"""Builds the sm_100a backend in-tree: every ``csrc/*.cu`` is compiled with
nvcc for ``compute_100a``/``sm_100a`` and linked into
``beatlm_b200/libbeatlm_b200.so`` (static CUDA runtime). The objects live in
``beatlm_b200/_build``. Nothing here needs a GPU; nvcc cross-compiles.

    python -m beatlm_b200.build [--force] [--verbose]
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
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libbeatlm_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
          "-Xcompiler", "-Wall", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _deps(src: str) -> list[str]:
    return [src] + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h")) \
        + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool, verbose: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    if force or _stale(obj, _deps(src)):
        cmd = [nvcc()] + ARCH + CFLAGS + (["-Xptxas", "-v"] if verbose else []) + \
            ["-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("nvcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
        if verbose and r.stderr:
            sys.stderr.write(r.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(BUILD, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, verbose), sources))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp%d" % os.getpid()
        cmd = [nvcc()] + ARCH + ["-shared", "-o", tmp] + objs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n%s%s" % (r.stdout, r.stderr))
        os.replace(tmp, LIB)
    return LIB


C_HOST = os.path.join(HERE, "c_host")


def build_c_host(force: bool = False) -> str:
    """The C-ABI-only host program ``c_host/vit_block.c`` (gcc, linked
    against the library, found beside it at run time), as
    ``_build/vit_block``; builds the library first."""
    lib = build(force)
    src = os.path.join(C_HOST, "vit_block.c")
    exe = os.path.join(BUILD, "vit_block")
    if force or _stale(exe, [src, lib, os.path.join(INCLUDE, "beatlm_b200.h")]):
        cmd = ["gcc", "-O2", "-std=c11", "-Wall", "-I", INCLUDE, src, "-o", exe + ".tmp",
               "-L", HERE, "-lbeatlm_b200", "-Wl,-rpath,$ORIGIN/..", "-lm"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("gcc failed for %s:\n%s%s" % (src, r.stdout, r.stderr))
        os.replace(exe + ".tmp", exe)
    return exe


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.verbose))
    print(build_c_host(a.force))
