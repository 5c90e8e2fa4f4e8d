"""Build ``libqx_b200.so`` (the C-ABI library) from ``csrc/*.cu`` with nvcc.

    python -m qextract_infer_b200.build [--force] [--verbose] [--trace]

Compiles every ``.cu`` file for sm_100a only (``-gencode
arch=compute_100a,code=sm_100a``) into ``_build/*.o`` and links the shared
library next to this file, so it travels with the source tree.  Objects are
rebuilt when their source or any header is newer.

``--trace`` builds the profiling library ``libqx_b200_trace.so`` instead
(objects in ``_build_trace/``, compiled with ``-DQX_TRACE``): the same kernels
with per-CTA phase timestamps, recorded when ``qx_trace_launches`` is given a
buffer (``bench.py --workload timeline`` reads them).  The package never loads
it; the product library carries no trace code.
"""

from __future__ import annotations

import argparse
import glob
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libqx_b200.so")
BUILD_TRACE = os.path.join(PKG, "_build_trace")
LIB_TRACE = os.path.join(PKG, "libqx_b200_trace.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(cand):
        raise RuntimeError("nvcc not found (CUDA toolkit required to build libqx_b200.so)")
    return cand


def _headers():
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _stale(out, deps):
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def build(force: bool = False, verbose: bool = False, extra_flags=None, trace: bool = False) -> str:
    build_dir, lib = (BUILD_TRACE, LIB_TRACE) if trace else (BUILD, LIB)
    os.makedirs(build_dir, exist_ok=True)
    srcs = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    hdrs = _headers()
    flags = NVCC_FLAGS + list(extra_flags or []) + (["-DQX_TRACE"] if trace else [])
    nv = nvcc()

    def compile_one(src):
        obj = os.path.join(build_dir, os.path.basename(src)[:-3] + ".o")
        if force or _stale(obj, [src] + hdrs):
            cmd = [nv, *ARCH, *flags, "-c", src, "-o", obj]
            if verbose:
                print(" ".join(cmd), flush=True)
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
            if verbose and (r.stdout or r.stderr):
                print(r.stdout + r.stderr, flush=True)
        return obj

    with ThreadPoolExecutor(max_workers=min(8, len(srcs) or 1)) as ex:
        objs = list(ex.map(compile_one, srcs))
    if force or _stale(lib, objs):
        tmp = lib + f".tmp{os.getpid()}"
        cmd = [nv, *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, lib)
    return lib


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--trace", action="store_true", help="build the profiling library libqx_b200_trace.so")
    a = ap.parse_args(argv)
    print(build(force=a.force, verbose=a.verbose, trace=a.trace))


if __name__ == "__main__":
    main(sys.argv[1:])
