"""The llama2 matmul offload without a GPU: struct layout, the exported
entry points and the C++ vxmath API, the oracle against numpy, and the oracle
pinned to the reference's own CPU matmul through its unchanged llama.cpp and
vxmath.cpp (benchmarks/llama2) running on the host-memory Vortex device."""
import ctypes as C
import os
import subprocess

import numpy as np
import pytest

from akili_bench_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PIN = os.path.join(ROOT, "oracle", "_ref", "pin")
VXMATH_LIB = os.path.join(ROOT, "akili_bench_b200", "libakili_vxmath.so")
TOKENS = [1, 300, 45, 67, 89, 120, 7, 333, 400, 12, 5, 77, 260, 261, 500, 3]


def test_matmul_kernel_args_layout():
    # benchmarks/llama2/common.h:3-12 on x86-64 / RV64
    assert C.sizeof(abi.MatmulKernelArgs) == 56
    assert abi.MatmulKernelArgs.A_addr.offset == 16 and abi.MatmulKernelArgs.C_addr.offset == 32
    assert abi.MatmulKernelArgs.M.offset == 40 and abi.MatmulKernelArgs.K.offset == 48
    assert C.sizeof(abi.MatvecSeg) == 24


def test_vxmath_library_exports_the_reference_api():
    """libakili_vxmath.so defines llama2/vxmath.h's five functions with the
    C++ signatures llama.cpp calls."""
    out = subprocess.run(["nm", "-D", "--defined-only", VXMATH_LIB], capture_output=True, text=True,
                         check=True).stdout
    syms = {ln.split()[-1] for ln in out.splitlines() if " T " in ln}
    assert {"_Z7vx_initv", "_Z9vx_matmulPfS_S_iii", "_Z14matmul_cleanupv",
            "_Z19vx_matmul_qkv_batchPfS_S_S_S_S_S_ii", "_Z19vx_matmul_ffn_batchPfS_S_S_S_ii"} <= syms
    C.CDLL(VXMATH_LIB)


def test_llama2_entries_validate_before_cuda():
    L = abi.load()
    assert L.akili_llama2_matmul(None, None) == abi.E_NULL_ARG
    a = abi.MatmulKernelArgs()
    a.M, a.N, a.K = -1, 1, 4
    assert L.akili_llama2_matmul(C.byref(a), None) == abi.E_SHAPE
    a.M, a.N, a.K = 0, 1, 4  # nothing to compute
    assert L.akili_llama2_matmul(C.byref(a), None) == abi.OK
    a.M, a.N, a.K, a.A_addr, a.B_addr, a.C_addr = 4, 1, 4, 16, 16, 0
    assert L.akili_llama2_matmul(C.byref(a), None) == abi.E_NULL_ARG
    a.C_addr = 18
    assert L.akili_llama2_matmul(C.byref(a), None) == abi.E_ALIGN
    segs = (abi.MatvecSeg * 5)()
    assert L.akili_llama2_matvec_batch(segs, 5, 16, 4, None) == abi.E_UNSUPPORTED
    assert L.akili_llama2_matvec_batch(segs, 0, 16, 4, None) == abi.E_UNSUPPORTED
    assert L.akili_llama2_matvec_batch(None, 1, 16, 4, None) == abi.E_NULL_ARG
    segs[0].rows = -2
    assert L.akili_llama2_matvec_batch(segs, 1, 16, 4, None) == abi.E_SHAPE


@pytest.mark.parametrize("M,N,K", [(7, 1, 13), (64, 1, 288), (5, 3, 9), (16, 8, 24)])
def test_oracle_matmul_against_numpy(oracle, M, N, K):
    rng = np.random.default_rng(M * N + K)
    a = rng.standard_normal((M, K), dtype=np.float32)
    b = rng.standard_normal((K, N), dtype=np.float32)
    got = oracle.llama2_matmul(a, b, M, N, K)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    assert np.abs(got - ref).max() <= 1e-5 * (np.abs(a) @ np.abs(b)).max()


def _model(tmp_path):
    import sys
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_llama2_model as mk
    return mk.write_model(str(tmp_path), "tiny", seed=0)


def _run(exe, *args, env_op=True):
    env = dict(os.environ, AKILI_OP="llama2_matmul") if env_op else None
    return subprocess.run([exe, *map(str, args)], capture_output=True, text=True, timeout=120, env=env)


@pytest.mark.skipif(not os.path.exists(os.path.join(PIN, "llama2_logits")),
                    reason="oracle/_ref not built (needs the reference tree)")
def test_oracle_pinned_to_reference_llama_cpu_path(tmp_path):
    """Every position's logits from llama.cpp with the reference's CPU matmul
    (-v 0) and with its vxmath.cpp offload running the oracle (-v 1) are
    identical bit for bit: the oracle restates the reference matmul exactly,
    batched QKV/FFN concatenation included."""
    ckpt, _ = _model(tmp_path)
    outs = []
    for v in (0, 1):
        out = tmp_path / f"logits{v}.bin"
        r = _run(os.path.join(PIN, "llama2_logits"), ckpt, v, out, *TOKENS)
        assert r.returncode == 0, r.stderr
        outs.append(np.fromfile(out, np.float32))
    assert outs[0].size == len(TOKENS) * 512
    assert np.array_equal(outs[0], outs[1])
    assert np.isfinite(outs[0]).all() and np.abs(outs[0]).max() > 0.1


@pytest.mark.skipif(not os.path.exists(os.path.join(PIN, "llama")), reason="oracle/_ref not built")
def test_reference_llama_generates_the_same_text_on_the_oracle(tmp_path):
    ckpt, tok = _model(tmp_path)
    texts = []
    for v in (0, 1):
        r = _run(os.path.join(PIN, "llama"), ckpt, "-z", tok, "-t", 0, "-n", 40, "-i", "the cat", "-v", v)
        assert r.returncode == 0, r.stderr
        texts.append(r.stdout.replace(">> Using vortex acceleration\n", "").replace("open device connection\n", ""))
    assert texts[0] == texts[1]
    assert texts[0].startswith("the cat") and len(texts[0]) > 20
