"""Build ``libspecdec_b200.so`` in-tree with nvcc for sm_100a.

    python specdec-nanovllm_b200/build.py [--force] [--verbose]

Each ``csrc/*.cu`` compiles to an object in ``_build/`` (in parallel), then one
shared library links them with the shared CUDA runtime, so the library and torch
share the same runtime state (current device, streams).  Rebuilds only what is
older than its sources.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libspecdec_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-I", INCLUDE,
                     "-I", CSRC, "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _deps():
    hdrs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    hdrs += [os.path.join(INCLUDE, f) for f in os.listdir(INCLUDE)]
    return max((os.path.getmtime(h) for h in hdrs), default=0.0)


def _compile(src: str, force: bool, verbose: bool, extra):
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    newest = max(os.path.getmtime(src), _deps())
    if not force and os.path.exists(obj) and os.path.getmtime(obj) >= newest:
        return obj, ""
    cmd = [nvcc()] + NVCC_FLAGS + list(extra) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj, (r.stdout + r.stderr) if verbose else ""


def build(force: bool = False, verbose: bool = False, extra=()) -> str:
    os.makedirs(BUILD, exist_ok=True)
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, force, verbose, extra), srcs))
    objs = [o for o, _ in results]
    for _, log in results:
        if log:
            print(log, file=sys.stderr)
    if force or not os.path.exists(LIB) or os.path.getmtime(LIB) < max(os.path.getmtime(o) for o in objs):
        cuda_lib = os.path.join(os.path.dirname(os.path.dirname(nvcc())), "lib64")
        cmd = [nvcc()] + ARCH + ["-shared", "-cudart", "shared", "-o", LIB] + objs + \
              ["-Xlinker", f"-rpath={cuda_lib}"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas resource usage")
    a = ap.parse_args()
    extra = ["-Xptxas", "-v"] if a.verbose else []
    print(build(force=a.force or a.verbose, verbose=a.verbose, extra=extra))
