"""Build the in-tree native libraries for sm_100a.

    python -m akili_bench_b200.build        (or akili_bench_b200.build.build())

* ``libakili.so``        csrc/akili.cu — every kernel and the C ABI of
                         include/akili.h (nvcc, -gencode arch=compute_100a,
                         code=sm_100a, static cudart; the driver API is reached
                         through cudaGetDriverEntryPoint, so loading needs no
                         libcuda until the first call).
* ``libakili_vortex.so`` csrc/vortex_shim.cpp — the Vortex runtime API of
                         include/vortex.h on top of libakili.so, for
                         akili-bench's unchanged host harnesses.
* ``libakili_vxmath.so`` csrc/vxmath_b200.cpp — the llama2 matmul offload
                         API (benchmarks/llama2/vxmath.h) on top of
                         libakili.so, for the unchanged llama2/llama.cpp.

All land next to this file so they travel with the working tree.
"""
from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
if not os.path.exists(NVCC):
    NVCC = "nvcc"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-shared", "--expt-relaxed-constexpr",
              "-cudart", "static", "-I", os.path.join(ROOT, "include")]

LIB = os.path.join(HERE, "libakili.so")
VORTEX_LIB = os.path.join(HERE, "libakili_vortex.so")
VXMATH_LIB = os.path.join(HERE, "libakili_vxmath.so")


def _sources():
    return [os.path.join(CSRC, f) for f in sorted(os.listdir(CSRC)) if f.endswith((".cu", ".cuh"))] + \
        [os.path.join(ROOT, "include", "akili.h")]


def _stale(out: str, deps: list[str]) -> bool:
    if not os.path.exists(out):
        return True
    t = os.path.getmtime(out)
    return any(os.path.getmtime(d) > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build(force: bool = False, verbose: bool = False) -> list[str]:
    deps = _sources()
    if force or _stale(LIB, deps):
        cmd = [NVCC, *ARCH, *NVCC_FLAGS, os.path.join(CSRC, "akili.cu"), "-o", LIB]
        if verbose:
            print(" ".join(cmd))
        _run(cmd)
    cuda_inc = os.path.join(os.path.dirname(os.path.dirname(os.path.realpath(NVCC))), "include") \
        if os.path.isabs(NVCC) else "/usr/local/cuda/include"
    cuda_lib = os.path.join(os.path.dirname(cuda_inc), "lib64")
    for src, out, hdr in (("vortex_shim.cpp", VORTEX_LIB, "vortex.h"), ("vxmath_b200.cpp", VXMATH_LIB, "akili.h")):
        hdeps = [os.path.join(CSRC, src), os.path.join(ROOT, "include", hdr), LIB]
        if force or _stale(out, hdeps):
            cmd = ["g++", "-std=c++17", "-O2", "-fPIC", "-shared", "-I", os.path.join(ROOT, "include"), "-I",
                   cuda_inc, os.path.join(CSRC, src), "-o", out, "-L", HERE, "-lakili", f"-Wl,-rpath,{HERE}", "-L",
                   cuda_lib, "-lcudart_static", "-ldl", "-lpthread", "-lrt"]
            if verbose:
                print(" ".join(cmd))
            _run(cmd)
    return [LIB, VORTEX_LIB, VXMATH_LIB]


if __name__ == "__main__":
    for p in build(force="--force" in sys.argv, verbose=True):
        print(p)
