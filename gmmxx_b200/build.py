"""Build the engine's CUDA shared library (sm_100a only), in-tree.

    python -m gmmxx_b200.build            # incremental
    python -m gmmxx_b200.build --force    # rebuild everything

Each ``csrc/*.cu`` is compiled by nvcc (``-gencode arch=compute_100a,code=sm_100a``)
into ``_build/`` and linked into ``gmmxx_b200/_lib/libgmmxx_b200.so``; the C ABI
it exports is declared in ``include/gmmxx_b200.h``.  nvcc cross-compiles, so the
build needs no GPU.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
BUILD = os.path.join(ROOT, "_build")
LIBDIR = os.path.join(PKG, "_lib")
LIB = os.path.join(LIBDIR, "libgmmxx_b200.so")
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
          "--expt-relaxed-constexpr", "-DNDEBUG"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found; set NVCC or install the CUDA toolkit")


def _deps(src: str):
    deps = [src, os.path.join(INCLUDE, "gmmxx_b200.h")]
    deps += glob.glob(os.path.join(CSRC, "*.cuh"))
    return deps


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force: bool = False, verbose: bool = False, ptxas_verbose: bool = False) -> str:
    """Compile every csrc/*.cu and link the shared library; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIBDIR, exist_ok=True)
    nvcc = _nvcc()
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    objs = []
    jobs = []
    for src in srcs:
        obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
        objs.append(obj)
        if force or _stale(obj, _deps(src)):
            cmd = [nvcc, *ARCH, *CFLAGS, "-I", INCLUDE, "-c", src, "-o", obj]
            if ptxas_verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append((src, cmd))

    def run(job):
        src, cmd = job
        if verbose:
            print(" ".join(cmd), flush=True)
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {os.path.basename(src)}:\n{p.stdout}\n{p.stderr}")
        if ptxas_verbose or verbose:
            sys.stdout.write(p.stdout + p.stderr)
        return src

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [nvcc, *ARCH, "-shared", "-o", tmp, *objs, "-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        p = subprocess.run(cmd, capture_output=True, text=True)
        if p.returncode != 0:
            raise RuntimeError(f"link failed:\n{p.stdout}\n{p.stderr}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="print ptxas register / smem usage")
    args = ap.parse_args(argv)
    print(build(force=args.force, verbose=args.verbose, ptxas_verbose=args.ptxas))


if __name__ == "__main__":
    main()
