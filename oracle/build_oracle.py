"""Build recipe for the CPU oracle and the reference-built pin binaries.

TEST INFRASTRUCTURE.  Outputs:

* ``oracle/liboracle.so`` — oracle/oracle.c (the plain-C restatement of the
  reference gold loops), loaded by tests/ and by bench.py's CPU-baseline leg.
* ``oracle/_ref/pin/<bench>`` — akili-bench's own, unchanged
  ``benchmarks/<bench>/main.cpp`` compiled with the reference's host flags
  (common/common.mk:63-71: ``-std=c++17 -O2 -DNDEBUG``) against
  ``include/vortex.h`` + ``oracle/shim/vortex_host.cpp`` (a host-memory
  device that runs the oracle) and force-including ``oracle/shim/probe.h``.
  Run with ``AKILI_PROBE=exact`` the reference's verify loop passes only if
  the oracle is bit-identical to the reference gold.
* ``oracle/_ref/b200/<bench>`` — the same unchanged ``main.cpp`` linked
  against the product's ``libakili_vortex.so`` (the Vortex runtime API on
  top of the akili_* C ABI): the reference harness driving the B200 kernels
  and judging them with its own gold check.
* llama2 (``benchmarks/llama2``: the reference's ``llama.cpp`` and its
  matmul offload ``vxmath.cpp``, unchanged):
  ``oracle/_ref/pin/llama`` and ``oracle/_ref/pin/llama2_logits`` over the
  host-memory device (``-v 0`` is the reference's CPU matmul, ``-v 1`` its
  vxmath.cpp driving the oracle); ``oracle/_ref/b200/llama`` and
  ``.../llama2_logits`` with vxmath.cpp over ``libakili_vortex.so``;
  ``oracle/_ref/b200/llama_vxmath`` and ``.../llama2_logits_vxmath`` with
  the product's ``libakili_vxmath.so`` in place of vxmath.cpp.
  ``llama2_logits`` is ``oracle/llama2/llama2_logits.cpp``, a driver that
  compiles llama.cpp with TESTING and writes each position's logits.
* ``oracle/_ref/libdao_flash_ref.so`` — the CuPBoP causal flash benchmark
  ``benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu`` (plain CUDA: its CPU
  gold ``attention_cpu`` and its kernel ``dao_flash_fwd``), compiled by nvcc
  through ``oracle/shim/dao_flash_ref.cu``, which gives both C entry points.
  It pins the causal flash oracle and the m / l row statistics.

The reference sources are read in place (``--ref``, or the
``AKILI_REFERENCE_ROOT`` environment variable); nothing is copied.  ``oracle/_ref/`` is git-ignored and
travels with the working tree like the other built artefacts.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
REF_OUT = os.path.join(HERE, "_ref")

BENCHES = [
    "kbt_sgemm",
    "kbt_gemm_add_relu",
    "kbt_gemm_mul_leakyrelu",
    "kbt_gemm_div_sum_scale",
    "kbt_gemm_layernorm",
    "kbt_attention_score",
    "kbt_matmul_softmax",
    "kbt_matmul_scale_residadd_clamp",
    "kbt_matmul_sum_max_avgpool",
    "kbt_gemm_rmsnorm_swiglu",
    "kbt_gemm_silu_mul",
    "flash",
    "attention",
    "kb2_gemm_add_relu",
    "kb2_gemm_mul_leakyrelu",
    "kb2_gemm_div_sum_scale",
    "kb2_gemm_layernorm",
    "kb2_attention_score",
    "kb2_matmul_softmax",
    "kb2_matmul_scale_residadd_clamp",
    "kb2_matmul_sum_max_avgpool",
    "kb2_gemm_rmsnorm_swiglu",
    "kb2_gemm_silu_mul",
]

# The reference's host compile flags (common/common.mk:63,69-71).
REF_CXXFLAGS = ["-std=c++17", "-O2", "-DNDEBUG"]
# The oracle is compiled with the same optimisation level and no FMA ISA so
# its float arithmetic matches the reference's gold loops bit for bit.
ORACLE_CFLAGS = ["-std=c11", "-O2", "-DNDEBUG", "-fPIC", "-ffp-contract=off"]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _newer(out: str, srcs: list[str]) -> bool:
    if not os.path.exists(out):
        return False
    t = os.path.getmtime(out)
    return all(os.path.getmtime(s) <= t for s in srcs if os.path.exists(s))


def build_oracle_lib(force: bool = False) -> str:
    """Compile oracle/oracle.c into oracle/liboracle.so."""
    src = os.path.join(HERE, "oracle.c")
    out = os.path.join(HERE, "liboracle.so")
    if force or not _newer(out, [src, os.path.join(HERE, "oracle.h")]):
        _run(["gcc", *ORACLE_CFLAGS, "-shared", src, "-o", out, "-lm"])
    return out


def build_pin_binaries(ref_root: str, force: bool = False) -> list[str]:
    """Reference main.cpp + host-memory Vortex device running the oracle."""
    os.makedirs(os.path.join(REF_OUT, "pin"), exist_ok=True)
    obj = os.path.join(REF_OUT, "oracle_pin.o")
    _run(["gcc", *ORACLE_CFLAGS, "-c", os.path.join(HERE, "oracle.c"), "-o", obj])
    shim = os.path.join(HERE, "shim", "vortex_host.cpp")
    probe = os.path.join(HERE, "shim", "probe.h")
    # The shim is its own translation unit: the probe macros apply to main.cpp only.
    shim_obj = os.path.join(REF_OUT, "vortex_host.o")
    _run(["g++", *REF_CXXFLAGS, "-ffp-contract=off", "-I", os.path.join(ROOT, "include"),
          "-c", shim, "-o", shim_obj])
    built = []
    for b in BENCHES:
        main = os.path.join(ref_root, "benchmarks", b, "main.cpp")
        out = os.path.join(REF_OUT, "pin", b)
        if not force and _newer(out, [main, shim, probe, obj]):
            built.append(out)
            continue
        _run(["g++", *REF_CXXFLAGS, "-ffp-contract=off", "-I", os.path.join(ROOT, "include"),
              "-include", probe, main, shim_obj, obj, "-o", out, "-lm"])
        built.append(out)
    return built


def build_b200_binaries(ref_root: str, libdir: str, force: bool = False) -> list[str]:
    """Reference main.cpp linked against the product's Vortex-API library."""
    lib = os.path.join(libdir, "libakili_vortex.so")
    if not os.path.exists(lib):
        raise FileNotFoundError(lib)
    os.makedirs(os.path.join(REF_OUT, "b200"), exist_ok=True)
    built = []
    for b in BENCHES:
        main = os.path.join(ref_root, "benchmarks", b, "main.cpp")
        out = os.path.join(REF_OUT, "b200", b)
        if not force and _newer(out, [main, lib]):
            built.append(out)
            continue
        _run(["g++", *REF_CXXFLAGS, "-I", os.path.join(ROOT, "include"), main,
              "-L", libdir, "-lakili_vortex", f"-Wl,-rpath,{libdir}", "-o", out])
        built.append(out)
    return built


def build_llama2_binaries(ref_root: str, libdir: str, force: bool = False) -> list[str]:
    """The reference llama2 program (and the logits driver) against the
    host-memory device, the product's Vortex shim and its vxmath library."""
    src_dir = os.path.join(ref_root, "benchmarks", "llama2")
    llama = os.path.join(src_dir, "llama.cpp")
    vxmath = os.path.join(src_dir, "vxmath.cpp")
    driver = os.path.join(HERE, "llama2", "llama2_logits.cpp")
    inc = ["-I", os.path.join(ROOT, "include"), "-I", src_dir]
    flags = [*REF_CXXFLAGS, "-ffp-contract=off", "-w"]
    built = []
    pin_objs = [os.path.join(REF_OUT, "vortex_host.o"), os.path.join(REF_OUT, "oracle_pin.o")]
    os.makedirs(os.path.join(REF_OUT, "pin"), exist_ok=True)
    for name, main_src in (("llama", llama), ("llama2_logits", driver)):
        out = os.path.join(REF_OUT, "pin", name)
        deps = [main_src, llama, vxmath, *pin_objs]
        if force or not _newer(out, deps):
            _run(["g++", *flags, *inc, main_src, vxmath, *pin_objs, "-o", out, "-lm"])
        built.append(out)
    vortex_lib = os.path.join(libdir, "libakili_vortex.so")
    vxmath_lib = os.path.join(libdir, "libakili_vxmath.so")
    os.makedirs(os.path.join(REF_OUT, "b200"), exist_ok=True)
    for name, main_src, extra, lib in (
            ("llama", llama, [vxmath], "akili_vortex"),
            ("llama2_logits", driver, [vxmath], "akili_vortex"),
            ("llama_vxmath", llama, [], "akili_vxmath"),
            ("llama2_logits_vxmath", driver, [], "akili_vxmath")):
        libpath = vortex_lib if lib == "akili_vortex" else vxmath_lib
        if not os.path.exists(libpath):
            continue
        out = os.path.join(REF_OUT, "b200", name)
        if force or not _newer(out, [main_src, llama, *extra, libpath]):
            _run(["g++", *flags, *inc, main_src, *extra, "-L", libdir, f"-l{lib}", f"-Wl,-rpath,{libdir}", "-o",
                  out, "-lm"])
        built.append(out)
    return built


def build_dao_flash_ref(ref_root: str, force: bool = False) -> str:
    """benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu, unchanged, as a
    shared library with C entry points (oracle/shim/dao_flash_ref.cu)."""
    src_dir = os.path.join(ref_root, "benchmarks", "cupbop_dao_flash")
    wrapper = os.path.join(HERE, "shim", "dao_flash_ref.cu")
    out = os.path.join(REF_OUT, "libdao_flash_ref.so")
    os.makedirs(REF_OUT, exist_ok=True)
    if force or not _newer(out, [wrapper, os.path.join(src_dir, "dao_flash_cupbop.cu")]):
        nvcc = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
        if not os.path.exists(nvcc):
            nvcc = "nvcc"
        # host code: the reference's -O2 and, like the oracle, no FMA contraction
        _run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-std=c++17", "-shared",
              "-Xcompiler", "-fPIC,-ffp-contract=off", "-I", src_dir, "-Dmain=akili_ref_dao_main", wrapper,
              "-o", out])
    return out


# Where this recipe reads the reference tree when neither --ref nor
# $AKILI_REFERENCE_ROOT names one: the read-only checkout of the build
# container.  GPU boxes have no reference tree and use the prebuilt files.
DEFAULT_REFERENCE_ROOT = "/root/reference"


def reference_root(arg: str | None = None) -> str | None:
    """The reference tree: the argument, else $AKILI_REFERENCE_ROOT, else
    DEFAULT_REFERENCE_ROOT; None when that is not a directory."""
    ref = arg or os.environ.get("AKILI_REFERENCE_ROOT") or DEFAULT_REFERENCE_ROOT
    return ref if os.path.isdir(ref) else None


def main() -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ref", default=None,
                    help="reference tree (default: $AKILI_REFERENCE_ROOT, else DEFAULT_REFERENCE_ROOT)")
    ap.add_argument("--libdir", default=os.path.join(ROOT, "akili_bench_b200"))
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build_oracle_lib(a.force))
    ref = reference_root(a.ref)
    if ref:
        for p in build_pin_binaries(ref, a.force):
            print(p)
        if os.path.exists(os.path.join(a.libdir, "libakili_vortex.so")):
            for p in build_b200_binaries(ref, a.libdir, a.force):
                print(p)
        for p in build_llama2_binaries(ref, a.libdir, a.force):
            print(p)
        print(build_dao_flash_ref(ref, a.force))
    else:
        print("no reference tree: pin binaries not rebuilt", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
