"""Builds libproxima_b200.so (all CUDA sources under csrc/) for sm_100a.

Usage: python -m proxima_b200.build [--force] [--verbose]

The library is built in-tree (proxima_b200/libproxima_b200.so) so that it
travels with the repository to a GPU host. The CUDA runtime is linked
statically, so the library does not depend on whichever libcudart another
package (e.g. torch) loaded first.
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
OUT = os.path.join(HERE, "libproxima_b200.so")
OBJ = os.path.join(ROOT, "_build", "obj")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-fvisibility=hidden,-O3",
    "-I", os.path.join(ROOT, "include"),
]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def _sources():
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps():
    return _sources() + glob.glob(os.path.join(CSRC, "*.h")) + glob.glob(os.path.join(CSRC, "*.cuh")) + [
        os.path.join(ROOT, "include", "px.h")]


def up_to_date() -> bool:
    if not os.path.exists(OUT):
        return False
    t = os.path.getmtime(OUT)
    return all(os.path.getmtime(p) <= t for p in _deps())


def build(force: bool = False, verbose: bool = False, extra_flags=None) -> str:
    if not force and up_to_date():
        return OUT
    os.makedirs(OBJ, exist_ok=True)
    cc = nvcc()
    flags = NVCC_FLAGS + list(extra_flags or [])

    def compile_one(src):
        obj = os.path.join(OBJ, os.path.basename(src) + ".o")
        cmd = [cc] + flags + ["-c", src, "-o", obj]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout + r.stderr, flush=True)
        return obj

    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(compile_one, _sources()))
    tmp = OUT + ".tmp"
    cmd = [cc] + ARCH + ["-shared", "-cudart", "static", "-o", tmp] + objs + ["-ldl", "-lpthread"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, OUT)
    return OUT


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-v", action="store_true", help="print register/smem usage")
    a = ap.parse_args(argv)
    extra = ["-Xptxas", "-v"] if a.ptxas_v else None
    print(build(force=a.force or a.ptxas_v, verbose=a.verbose or a.ptxas_v, extra_flags=extra))


if __name__ == "__main__":
    sys.exit(main())
