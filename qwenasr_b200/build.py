"""Build libqwenasr_b200.so in-tree with nvcc for sm_100a.

    python -m qwenasr_b200.build [--force] [--verbose]

Each .cu under csrc/ is compiled to an object in csrc/_build/ (in parallel),
then linked into qwenasr_b200/libqwenasr_b200.so.  --fmad=false keeps nvcc
from contracting a*b+c into FMAs the source did not ask for (the kernels
reproduce the reference's rounding sequence); -ffp-contract=off does the same
for host code (the log-mel tables are built on the host).  No GPU is needed
to build.
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(HERE, "libqwenasr_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "--fmad=false", "-std=c++17", "-Xcompiler", "-fPIC",
                     "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-ffp-contract=off", "--expt-relaxed-constexpr", f"-I{INCLUDE}"]


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _headers():
    return sorted(glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target, deps):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    hdrs = _headers()
    flags = NVCC_FLAGS + list(extra_flags or [])
    objs = []
    jobs = []
    for s in srcs:
        o = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        objs.append(o)
        if force or _stale(o, [s] + hdrs + [__file__]):
            jobs.append([NVCC] + flags + ["-c", s, "-o", o])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {cmd[-3]}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)

    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
            list(ex.map(run, jobs))
    if force or jobs or _stale(LIB, objs):
        run([NVCC] + ARCH + ["-shared", "-o", LIB] + objs + ["-lcudart"])
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true", help="print -Xptxas -v register/spill report")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_info else []
    print(build(force=a.force or a.ptxas_info, verbose=a.verbose or a.ptxas_info, extra_flags=extra))


if __name__ == "__main__":
    sys.exit(main())
