"""Builds libdnb200.so, the sm_100a kernels plus their C ABI, in-tree.

    python -m darknet_zig_b200.build [--force]

Every .cu under csrc/ is compiled separately (in parallel) with
    nvcc -std=c++20 -gencode arch=compute_100a,code=sm_100a -O3 -lineinfo --fmad=false
and linked into darknet_zig_b200/libdnb200.so with the static CUDA runtime. --fmad=false
keeps every a*b+c as two roundings, as the reference's strict-mode CPU code computes it;
the kernels fuse explicitly (__fmaf_rn) only where the reference does (blas.axpy).
"""
from __future__ import annotations

import concurrent.futures as cf
import glob
import os
import shutil
import subprocess
import sys

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
OBJ = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "libdnb200.so")



def nvcc_path() -> str | None:
    """nvcc from $NVCC, else $CUDA_HOME / $CUDA_PATH, else the PATH; None if there is none."""
    if os.environ.get("NVCC"):
        return os.environ["NVCC"]
    for var in ("CUDA_HOME", "CUDA_PATH"):
        home = os.environ.get(var)
        if home and os.path.exists(os.path.join(home, "bin", "nvcc")):
            return os.path.join(home, "bin", "nvcc")
    return shutil.which("nvcc")


def find_nvcc() -> str:
    found = nvcc_path()
    if not found:
        raise RuntimeError("nvcc not found: set NVCC or CUDA_HOME, or put nvcc on the PATH")
    return found


ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-std=c++20", *ARCH, "-O3", "-lineinfo", "--fmad=false", "-Xcompiler", "-fPIC,-O2",
         "-I", INCLUDE, "-I", CSRC]


def _headers() -> list[str]:
    return glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))


def _newer(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, force: bool) -> str:
    obj = os.path.join(OBJ, os.path.basename(src)[:-3] + ".o")
    if force or _newer(obj, [src, __file__, *_headers()]):
        cmd = [find_nvcc(), *FLAGS, "-c", src, "-o", obj]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    os.makedirs(OBJ, exist_ok=True)
    sources = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force), sources))
    if force or _newer(LIB, objs):
        cmd = [find_nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", LIB, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
