"""numpy front end of the CPU oracle (oracle/oracle.c via ctypes).

TEST INFRASTRUCTURE: imported only by tests/, ``__graft_entry__.smoke()`` and
the CPU-baseline leg of bench.py.  Every function takes fp32 numpy arrays
(row-major), computes rows ``[row0, row1)`` and can split those rows over
``threads`` host threads (ctypes releases the GIL during each call; rows are
independent in every op, so the result does not depend on the split).
"""
from __future__ import annotations

import ctypes as C
import os
from concurrent.futures import ThreadPoolExecutor

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB = None

_f32p = C.POINTER(C.c_float)
_u32 = C.c_uint32
_f = C.c_float

_SIGS = {
    "oracle_kbt_sgemm": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kbt_gemm_add_relu": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kbt_gemm_mul_leakyrelu": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _f, _u32, _u32],
    "oracle_kbt_gemm_div_sum_scale": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kbt_gemm_layernorm": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kbt_attention_score": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kbt_matmul_softmax": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kbt_matmul_scale_residadd_clamp": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _f, _f, _u32, _u32],
    "oracle_kbt_matmul_sum_max_avgpool": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kbt_gemm_rmsnorm_swiglu": [_f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kbt_gemm_silu_mul": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_flash": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _f, _u32, _u32],
    "oracle_flash_causal": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _f, _u32, _u32, _u32],
    "oracle_kb2_gemm_add_relu": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kb2_gemm_mul_leakyrelu": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _f, _u32, _u32],
    "oracle_kb2_gemm_div_sum_scale": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kb2_gemm_layernorm": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kb2_attention_score": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kb2_matmul_softmax": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kb2_matmul_scale_residadd_clamp": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _f, _f, _u32,
                                               _u32],
    "oracle_kb2_matmul_sum_max_avgpool": [_f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_kb2_gemm_rmsnorm_swiglu": [_f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _f, _u32, _u32],
    "oracle_kb2_gemm_silu_mul": [_f32p, _f32p, _f32p, _f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_attention_matmul": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_attention_softmax": [_f32p, _f32p, _u32, _u32, _u32, _u32],
    "oracle_llama2_matmul": [_f32p, _f32p, _f32p, _u32, _u32, _u32, _u32, _u32],
    "oracle_round_f16_array": [_f32p, C.c_uint64],
}


def lib() -> C.CDLL:
    """Load oracle/liboracle.so, building it from oracle.c if it is missing."""
    global _LIB
    if _LIB is None:
        path = os.path.join(_HERE, "liboracle.so")
        if not os.path.exists(path):
            import importlib.util
            spec = importlib.util.spec_from_file_location("_akili_build_oracle",
                                                          os.path.join(_HERE, "build_oracle.py"))
            mod = importlib.util.module_from_spec(spec)
            spec.loader.exec_module(mod)  # type: ignore[union-attr]
            mod.build_oracle_lib()
        L = C.CDLL(path)
        for name, argt in _SIGS.items():
            fn = getattr(L, name)
            fn.argtypes = argt
            fn.restype = None
        _LIB = L
    return _LIB


def _p(x: np.ndarray):
    assert x.dtype == np.float32 and x.flags["C_CONTIGUOUS"], "oracle wants C-contiguous fp32"
    return x.ctypes.data_as(_f32p)


def _split(row0: int, row1: int, threads: int):
    n = row1 - row0
    threads = max(1, min(threads, n)) if n > 0 else 1
    step = (n + threads - 1) // threads if n > 0 else 0
    return [(row0 + i * step, min(row1, row0 + (i + 1) * step)) for i in range(threads) if row0 + i * step < row1]


def _rows(fn, args_before, args_after, row0, row1, threads):
    parts = _split(row0, row1, threads)
    if len(parts) <= 1:
        for a, b in parts:
            fn(*args_before, *args_after, a, b)
        return
    with ThreadPoolExecutor(len(parts)) as ex:
        list(ex.map(lambda ab: fn(*args_before, *args_after, ab[0], ab[1]), parts))


def round_f16(x: np.ndarray) -> np.ndarray:
    """fp32 -> fp16 (round to nearest even) -> fp32, in a copy."""
    y = np.ascontiguousarray(x, dtype=np.float32).copy()
    lib().oracle_round_f16_array(_p(y), y.size)
    return y


def _out(shape, out):
    return np.zeros(shape, np.float32) if out is None else out


def kbt_sgemm(a, b, M, N, K, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_sgemm, (_p(a), _p(b), _p(c)), (M, N, K), row0, row1, threads)
    return c


def kbt_gemm_add_relu(a, w, bias, M, N, K, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_gemm_add_relu, (_p(a), _p(w), _p(bias), _p(c)), (M, N, K), row0, row1, threads)
    return c


def kbt_gemm_mul_leakyrelu(a, w, bias, M, N, K, multiplier, negative_slope, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_gemm_mul_leakyrelu, (_p(a), _p(w), _p(bias), _p(c)),
          (M, N, K, multiplier, negative_slope), row0, row1, threads)
    return c


def kbt_gemm_div_sum_scale(a, w, M, N, K, scaling_factor, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M,), out)
    _rows(lib().oracle_kbt_gemm_div_sum_scale, (_p(a), _p(w), _p(c)), (M, N, K, scaling_factor),
          row0, row1, threads)
    return c


def kbt_gemm_layernorm(a, w, bias, ln_w, ln_b, M, N, K, eps, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_gemm_layernorm, (_p(a), _p(w), _p(bias), _p(ln_w), _p(ln_b), _p(c)),
          (M, N, K, eps), row0, row1, threads)
    return c


def kbt_attention_score(q, k, M, N, D, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_attention_score, (_p(q), _p(k), _p(c)), (M, N, D), row0, row1, threads)
    return c


def kbt_matmul_softmax(a, b, M, N, K, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_matmul_softmax, (_p(a), _p(b), _p(c)), (M, N, K), row0, row1, threads)
    return c


def kbt_matmul_scale_residadd_clamp(a, b, M, N, K, scale_factor, clamp_min, clamp_max, row0=0, row1=None,
                                    threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M,), out)
    _rows(lib().oracle_kbt_matmul_scale_residadd_clamp, (_p(a), _p(b), _p(c)),
          (M, N, K, scale_factor, clamp_min, clamp_max), row0, row1, threads)
    return c


def kbt_matmul_sum_max_avgpool(a, w, bias, M, N, K, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M,), out)
    _rows(lib().oracle_kbt_matmul_sum_max_avgpool, (_p(a), _p(w), _p(bias), _p(c)), (M, N, K),
          row0, row1, threads)
    return c


def kbt_gemm_rmsnorm_swiglu(x, rms_w, wg, wu, M, N, K, eps, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_gemm_rmsnorm_swiglu, (_p(x), _p(rms_w), _p(wg), _p(wu), _p(c)),
          (M, N, K, eps), row0, row1, threads)
    return c


def kbt_gemm_silu_mul(a, wa, ba, wb, bb, M, N, K, row0=0, row1=None, threads=1, out=None):
    row1 = M if row1 is None else row1
    c = _out((M, N), out)
    _rows(lib().oracle_kbt_gemm_silu_mul, (_p(a), _p(wa), _p(ba), _p(wb), _p(bb), _p(c)), (M, N, K),
          row0, row1, threads)
    return c


def flash(q, k, v, seq_len, d, scale=1.0, row0=0, row1=None, threads=1, out=None):
    """One head: q/k/v [seq_len x d]."""
    row1 = seq_len if row1 is None else row1
    o = _out((seq_len, d), out)
    _rows(lib().oracle_flash, (_p(o), _p(q), _p(k), _p(v)), (seq_len, d, scale), row0, row1, threads)
    return o


def flash_causal(q, k, v, seq_len, d, scale=1.0, causal=True, row0=0, row1=None, threads=1):
    """One head with the optional causal mask; returns (o, m, l): o [seq_len x d]
    and the per-row softmax statistics m, l [seq_len] (rows outside
    [row0, row1) are zero)."""
    row1 = seq_len if row1 is None else row1
    o = _out((seq_len, d), None)
    m = np.zeros(seq_len, np.float32)
    l = np.zeros(seq_len, np.float32)
    _rows(lib().oracle_flash_causal, (_p(o), _p(m), _p(l), _p(q), _p(k), _p(v)),
          (seq_len, d, scale, 1 if causal else 0), row0, row1, threads)
    return o, m, l


# ---- the kb2_* family (fp32 gold loops, bias-first dot products) ----

def kb2_gemm_add_relu(a, w, bias, M, N, K, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_gemm_add_relu, (_p(a), _p(w), _p(bias), _p(c)), (M, N, K), row0, row1, threads)
    return c


def kb2_gemm_mul_leakyrelu(a, w, bias, M, N, K, multiplier=1.5, negative_slope=0.01, row0=0, row1=None,
                           threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_gemm_mul_leakyrelu, (_p(a), _p(w), _p(bias), _p(c)),
          (M, N, K, multiplier, negative_slope), row0, row1, threads)
    return c


def kb2_gemm_div_sum_scale(a, w, M, N, K, scaling_factor=2.0, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros(M, np.float32)
    _rows(lib().oracle_kb2_gemm_div_sum_scale, (_p(a), _p(w), _p(c)), (M, N, K, scaling_factor), row0, row1,
          threads)
    return c


def kb2_gemm_layernorm(a, w, bias, ln_w, ln_b, M, N, K, eps=1e-5, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_gemm_layernorm, (_p(a), _p(w), _p(bias), _p(ln_w), _p(ln_b), _p(c)), (M, N, K, eps),
          row0, row1, threads)
    return c


def kb2_attention_score(q, k, M, N, D, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_attention_score, (_p(q), _p(k), _p(c)), (M, N, D), row0, row1, threads)
    return c


def kb2_matmul_softmax(a, b, M, N, K, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_matmul_softmax, (_p(a), _p(b), _p(c)), (M, N, K), row0, row1, threads)
    return c


def kb2_matmul_scale_residadd_clamp(a, w, bias, M, N, K, scale_factor=2.0, clamp_min=-10.0, clamp_max=10.0,
                                    row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros(M, np.float32)
    _rows(lib().oracle_kb2_matmul_scale_residadd_clamp, (_p(a), _p(w), _p(bias), _p(c)),
          (M, N, K, scale_factor, clamp_min, clamp_max), row0, row1, threads)
    return c


def kb2_matmul_sum_max_avgpool(a, w, bias, M, N, K, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros(M, np.float32)
    _rows(lib().oracle_kb2_matmul_sum_max_avgpool, (_p(a), _p(w), _p(bias), _p(c)), (M, N, K), row0, row1,
          threads)
    return c


def kb2_gemm_rmsnorm_swiglu(x, rms_w, wg, wu, M, N, K, eps=1e-5, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_gemm_rmsnorm_swiglu, (_p(x), _p(rms_w), _p(wg), _p(wu), _p(c)), (M, N, K, eps), row0,
          row1, threads)
    return c


def kb2_gemm_silu_mul(a, wa, ba, wb, bb, M, N, K, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_kb2_gemm_silu_mul, (_p(a), _p(wa), _p(ba), _p(wb), _p(bb), _p(c)), (M, N, K), row0, row1,
          threads)
    return c


# ---- benchmarks/attention (unfused, fp32) ----

def attention_matmul(a, b, M, N, K, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_attention_matmul, (_p(c), _p(a), _p(b)), (M, N, K), row0, row1, threads)
    return c


def attention_softmax(a, M, N, row0=0, row1=None, threads=1):
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_attention_softmax, (_p(c), _p(a)), (M, N), row0, row1, threads)
    return c


# ---- benchmarks/llama2 (matmul offload, fp32) ----

def llama2_matmul(a, b, M, N, K, row0=0, row1=None, threads=1):
    """C[M x N] = A[M x K] . B[K x N] (llama2/matmul_kernel.cpp:15-22)."""
    row1 = M if row1 is None else row1
    c = np.zeros((M, N), np.float32)
    _rows(lib().oracle_llama2_matmul, (_p(c), _p(a), _p(b)), (M, N, K), row0, row1, threads)
    return c
