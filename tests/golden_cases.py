"""Load the committed golden cases and evaluate them with the oracle.

A case (tests/golden/<bench>__<tag>.npz, made by tests/golden/make_golden.py
from akili-bench's own harness) holds the harness inputs, its raw argument
block and the reference gold output.
"""
from __future__ import annotations

import ctypes as C
import glob
import os

import numpy as np

from akili_bench_b200 import abi

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def case_files(bench: str | None = None) -> list[str]:
    """Harness captures (make_golden.py); the dao_flash__ attention_cpu
    vectors (make_dao_flash_golden.py) carry no argument block and are read
    by their own test."""
    pat = f"{bench}__*.npz" if bench else "*__*.npz"
    return sorted(p for p in glob.glob(os.path.join(GOLDEN, pat))
                  if not os.path.basename(p).startswith("dao_flash__"))


def load_case(path: str):
    d = dict(np.load(path))
    bench = os.path.basename(path).split("__")[0]
    st, size = abi.OPS[bench]
    raw = d.pop("arg").tobytes()
    assert len(raw) == size == C.sizeof(st)
    arg = st.from_buffer_copy(raw)
    return bench, arg, d


def oracle_eval(oracle, bench: str, arg, d: dict, round_inputs: bool = False) -> np.ndarray:
    """Run the oracle on a case's inputs with the case's argument block."""
    g = {k: (oracle.round_f16(v) if round_inputs and v.ndim else v) for k, v in d.items()
         if k not in ("expected", "argv")}
    if bench == "flash":
        n, dd = arg.seq_len, arg.head_dim
        return oracle.flash(g["Q"], g["K"], g["V"], n, dd, 1.0).ravel()
    M, N = arg.M, arg.N
    K = arg.D if bench in ("kbt_attention_score", "kb2_attention_score") else arg.K
    if bench.startswith("kb2_"):
        return _kb2_eval(oracle, bench, arg, g, M, N, K).ravel()
    if bench == "kbt_sgemm":
        out = oracle.kbt_sgemm(g["a"], g["b"], M, N, K)
    elif bench == "kbt_gemm_add_relu":
        out = oracle.kbt_gemm_add_relu(g["a"], g["w"], g["bias"], M, N, K)
    elif bench == "kbt_gemm_mul_leakyrelu":
        out = oracle.kbt_gemm_mul_leakyrelu(g["a"], g["w"], g["bias"], M, N, K, arg.multiplier,
                                            arg.negative_slope)
    elif bench == "kbt_gemm_div_sum_scale":
        out = oracle.kbt_gemm_div_sum_scale(g["a"], g["w"], M, N, K, arg.scaling_factor)
    elif bench == "kbt_gemm_layernorm":
        out = oracle.kbt_gemm_layernorm(g["a"], g["w"], g["bias"], g["ln_w"], g["ln_b"], M, N, K, arg.eps)
    elif bench == "kbt_attention_score":
        out = oracle.kbt_attention_score(g["q"], g["k"], M, N, K)
    elif bench == "kbt_matmul_softmax":
        out = oracle.kbt_matmul_softmax(g["a"], g["b"], M, N, K)
    elif bench == "kbt_matmul_scale_residadd_clamp":
        out = oracle.kbt_matmul_scale_residadd_clamp(g["a"], g["b"], M, N, K, arg.scale_factor,
                                                     arg.clamp_min, arg.clamp_max)
    elif bench == "kbt_matmul_sum_max_avgpool":
        out = oracle.kbt_matmul_sum_max_avgpool(g["a"], g["w"], g["bias"], M, N, K)
    elif bench == "kbt_gemm_rmsnorm_swiglu":
        out = oracle.kbt_gemm_rmsnorm_swiglu(g["x"], g["rms_w"], g["wg"], g["wu"], M, N, K, arg.eps)
    elif bench == "kbt_gemm_silu_mul":
        out = oracle.kbt_gemm_silu_mul(g["a"], g["wa"], g["ba"], g["wb"], g["bb"], M, N, K)
    else:
        raise KeyError(bench)
    return out.ravel()


def _kb2_eval(oracle, bench, arg, g, M, N, K):
    if bench == "kb2_gemm_add_relu":
        return oracle.kb2_gemm_add_relu(g["a"], g["w"], g["bias"], M, N, K)
    if bench == "kb2_gemm_mul_leakyrelu":
        return oracle.kb2_gemm_mul_leakyrelu(g["a"], g["w"], g["bias"], M, N, K, arg.multiplier, arg.negative_slope)
    if bench == "kb2_gemm_div_sum_scale":
        return oracle.kb2_gemm_div_sum_scale(g["a"], g["w"], M, N, K, arg.scaling_factor)
    if bench == "kb2_gemm_layernorm":
        return oracle.kb2_gemm_layernorm(g["a"], g["w"], g["bias"], g["ln_w"], g["ln_b"], M, N, K, arg.eps)
    if bench == "kb2_attention_score":
        return oracle.kb2_attention_score(g["q"], g["k"], M, N, K)
    if bench == "kb2_matmul_softmax":
        return oracle.kb2_matmul_softmax(g["a"], g["b"], M, N, K)
    if bench == "kb2_matmul_scale_residadd_clamp":
        return oracle.kb2_matmul_scale_residadd_clamp(g["a"], g["w"], g["bias"], M, N, K, arg.scale_factor,
                                                      arg.clamp_min, arg.clamp_max)
    if bench == "kb2_matmul_sum_max_avgpool":
        return oracle.kb2_matmul_sum_max_avgpool(g["a"], g["w"], g["bias"], M, N, K)
    if bench == "kb2_gemm_rmsnorm_swiglu":
        return oracle.kb2_gemm_rmsnorm_swiglu(g["x"], g["rms_w"], g["wg"], g["wu"], M, N, K, arg.eps)
    if bench == "kb2_gemm_silu_mul":
        return oracle.kb2_gemm_silu_mul(g["a"], g["wa"], g["ba"], g["wb"], g["bb"], M, N, K)
    raise KeyError(bench)
