"""Build ``libsbfa.so`` (all CUDA sources under ``csrc/``) for sm_100a.

Compiles each ``csrc/*.cu`` to an object with nvcc in parallel, then links
one shared library next to this file.  Rebuilds only what changed
(sources are compared against their object, headers against everything).

``--debug`` builds ``libsbfa_debug.so`` instead, with ``SBFA_DEBUG_BOUNDS``:
every plan index and tile coordinate the kernels read is range-checked on
the device, and a value out of range is recorded in the status word
(``sbfa_device_status`` code 3) and clamped, so the access stays in bounds.
It is the stand-in for a memory checker (none can run on the target pool):
the odd-shape GPU tests run through it as well.

    python graph-kernel-injection_b200/build_native.py [--verbose-ptxas] [--force] [--debug]
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
BUILD_DEBUG = os.path.join(HERE, "_build_debug")
LIB_DEBUG = os.path.join(HERE, "libsbfa_debug.so")
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


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = True,
          debug: bool = False) -> str:
    build_dir, lib = (BUILD_DEBUG, LIB_DEBUG) if debug else (BUILD, LIB)
    os.makedirs(build_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    heads = _headers()
    extra = ["-Xptxas", "-v"] if verbose_ptxas else []
    if debug:
        extra.append("-DSBFA_DEBUG_BOUNDS")
    jobs = []
    for s in srcs:
        obj = os.path.join(build_dir, os.path.basename(s)[:-3] + ".o")
        if force or verbose_ptxas or _stale(obj, [s, *heads, __file__]):
            jobs.append((s, obj))
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            futs = {ex.submit(_compile, s, o, extra): s for s, o in jobs}
            for f in cf.as_completed(futs):
                log = f.result()
                if log and (verbose_ptxas or not quiet):
                    print(f"--- {os.path.basename(futs[f])}\n{log}", file=sys.stderr)
    objs = [os.path.join(build_dir, os.path.basename(s)[:-3] + ".o") for s in srcs]
    if force or jobs or _stale(lib, objs):
        tmp = lib + ".tmp"
        # cudart is linked statically; driver entry points (tensor maps) are
        # resolved at run time with cudaGetDriverEntryPoint, so the library
        # loads on hosts without a GPU driver.
        cmd = [nvcc(), *ARCH, "-shared", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
        os.replace(tmp, lib)
    return lib


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    ap.add_argument("--debug", action="store_true",
                    help="build libsbfa_debug.so with device-side bounds checks")
    a = ap.parse_args()
    print(build(force=a.force, verbose_ptxas=a.verbose_ptxas, quiet=False, debug=a.debug))
