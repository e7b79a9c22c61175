"""TEST INFRASTRUCTURE -- builds the CPU oracle and, where the reference tree is mounted,
the reference's own kernel source as a host-emulated library.

Outputs:
  oracle/_build/liboracle.so   C restatement of the reference CPU ops (ref_ops.c)
  oracle/_ref/libref_emulate.so  the reference's src/kernels/darknet_kernels.hip compiled
                               by g++ for the host through hip_host_shim.h (built only
                               when the reference tree is present; it then travels with
                               the repository snapshot like any other built .so)
  oracle/_ref/libref_gpu.so      the same kernel file compiled by nvcc for sm_100a with the
                               reference's own flags (build.zig:144-156), behind the
                               launchers of ref_gpu.cu: the reference's GPU path, run on the
                               B200 as the per-op GPU baseline (same build condition)

Flags: -O3 -march=x86-64-v3 (AVX2+FMA, portable across the container and the GPU box
hosts; -march=native could emit instructions another host lacks) and -ffp-contract=off,
so no multiply-add is fused behind the restatement's back.
"""
from __future__ import annotations

import json
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD = os.path.join(HERE, "_build")
REF_OUT = os.path.join(HERE, "_ref")
ORACLE_SO = os.path.join(BUILD, "liboracle.so")
REF_EMU_SO = os.path.join(REF_OUT, "libref_emulate.so")


def _reference_kernels() -> str:
    """The reference's kernel file: $DNB_REFERENCE_KERNELS, else src/kernels/darknet_kernels.hip
    under $DNB_REFERENCE_ROOT, else under the `reference_path` that BASELINE.json (the
    repository's build setting for the reference checkout) names. "" when none is set."""
    path = os.environ.get("DNB_REFERENCE_KERNELS")
    if path:
        return path
    root = os.environ.get("DNB_REFERENCE_ROOT")
    if not root:
        try:
            with open(os.path.join(os.path.dirname(HERE), "BASELINE.json")) as f:
                root = json.load(f).get("reference_path") or ""
        except (OSError, ValueError):
            root = ""
    return os.path.join(root, "src", "kernels", "darknet_kernels.hip") if root else ""


REFERENCE_KERNELS = _reference_kernels()

CFLAGS = ["-O3", "-march=x86-64-v3", "-ffp-contract=off", "-fno-fast-math", "-fPIC", "-shared"]


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build_oracle(force: bool = False) -> str:
    src = os.path.join(HERE, "ref_ops.c")
    hdr = os.path.join(HERE, "ref_ops.h")
    os.makedirs(BUILD, exist_ok=True)
    if force or _stale(ORACLE_SO, [src, hdr, __file__]):
        cmd = ["gcc", *CFLAGS, "-fopenmp", "-Wall", "-o", ORACLE_SO, src, "-lm"]
        subprocess.check_call(cmd)
    return ORACLE_SO


def build_ref_emulation(force: bool = False) -> str | None:
    """Compile the reference's own kernel file for the host. Returns None when the
    reference tree is not mounted (e.g. on the GPU box, which uses the prebuilt file)."""
    if not REFERENCE_KERNELS or not os.path.exists(REFERENCE_KERNELS):
        return REF_EMU_SO if os.path.exists(REF_EMU_SO) else None
    src = os.path.join(HERE, "ref_emulate.cpp")
    shim = os.path.join(HERE, "hip_host_shim.h")
    os.makedirs(REF_OUT, exist_ok=True)
    if force or _stale(REF_EMU_SO, [src, shim, REFERENCE_KERNELS, __file__]):
        cmd = ["g++", "-std=c++20", *CFLAGS, "-w", "-pthread", "-I", os.path.join(HERE, "shim"),
               f"-DDNB_REFERENCE_KERNELS=\"{REFERENCE_KERNELS}\"",
               "-o", REF_EMU_SO, src, "-lm"]
        subprocess.check_call(cmd)
    return REF_EMU_SO


REF_GPU_SO = os.path.join(REF_OUT, "libref_gpu.so")


def build_ref_gpu(force: bool = False) -> str | None:
    """Compile the reference's kernel file for the B200 (nvcc, sm_100a). The reference builds
    it with `nvcc -x cu -O3 -arch=...` (build.zig:144-156), so this keeps nvcc's default
    contraction and precision flags. Returns None when neither the reference tree nor a
    prebuilt file is present."""
    if not REFERENCE_KERNELS or not os.path.exists(REFERENCE_KERNELS):
        return REF_GPU_SO if os.path.exists(REF_GPU_SO) else None
    src = os.path.join(HERE, "ref_gpu.cu")
    os.makedirs(REF_OUT, exist_ok=True)
    if force or _stale(REF_GPU_SO, [src, REFERENCE_KERNELS, __file__]):
        home = os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or ""
        nvcc = os.environ.get("NVCC") or os.path.join(home, "bin", "nvcc")
        cmd = [nvcc if home or os.environ.get("NVCC") else "nvcc", "-x", "cu", "-O3",
               "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-Wno-deprecated-gpu-targets",
               "-shared", "-Xcompiler", "-fPIC", f"-DDNB_REFERENCE_KERNELS=\"{REFERENCE_KERNELS}\"",
               "-o", REF_GPU_SO, src]
        subprocess.check_call(cmd)
    return REF_GPU_SO


def build_all(force: bool = False) -> None:
    build_oracle(force)
    build_ref_emulation(force)
    build_ref_gpu(force)


if __name__ == "__main__":
    build_all(force="--force" in sys.argv)
    print(ORACLE_SO)
    print(REF_EMU_SO if os.path.exists(REF_EMU_SO) else "(reference emulation not built)")
    print(REF_GPU_SO if os.path.exists(REF_GPU_SO) else "(reference GPU kernels not built)")
