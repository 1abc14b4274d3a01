"""Build ``libsbfa.so`` (all CUDA sources under ``csrc/``) for sm_100a.

Compiles each ``csrc/*.cu`` to an object with nvcc in parallel, then links
one shared library next to this file.  Rebuilds only what changed
(sources are compared against their object, headers against everything).

    python graph-kernel-injection_b200/build_native.py [--verbose-ptxas] [--force]
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
LIB = os.path.join(HERE, "libsbfa.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC",
              "--expt-relaxed-constexpr", "-I", INCLUDE]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(target: str, deps) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, obj: str, extra) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {os.path.basename(src)}:\n{r.stderr}")
    return r.stderr


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    heads = _headers()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    jobs = []
    for s in srcs:
        obj = os.path.join(BUILD, os.path.basename(s)[:-3] + ".o")
        if force or verbose_ptxas or _stale(obj, [s, *heads, __file__]):
            jobs.append((s, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                log = f.result()
                if log and (verbose_ptxas or not quiet):
                    print(f"--- {os.path.basename(futs[f])}\n{log}", file=sys.stderr)
    objs = [os.path.join(BUILD, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        # cudart is linked statically; driver entry points (tensor maps) are
        # resolved at run time with cudaGetDriverEntryPoint, so the library
        # loads on hosts without a GPU driver.
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas, quiet=False))
