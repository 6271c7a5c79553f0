"""ctypes mirror of include/akili.h and the loader of libakili.so.

The argument blocks are the reference's ``kernel_arg_t`` layouts
(benchmarks/<bench>/common.h of akili-bench), byte for byte; ``OPS`` maps
each benchmark name to its struct, its buffer fields and its scalar fields.
``load()`` opens the in-tree ``libakili.so`` and declares every entry point;
it raises if the library is missing — there is no fallback path.
"""
from __future__ import annotations

import ctypes as C
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libakili.so")
VORTEX_LIB_PATH = os.path.join(_HERE, "libakili_vortex.so")

ABI_VERSION = 1
DTYPE_F32 = 0
DTYPE_F16 = 1

OK = 0
E_NULL_ARG = -1
E_SHAPE = -2
E_ALIGN = -3
E_DTYPE = -4
E_UNSUPPORTED = -5
E_NO_DEVICE = -6
E_ALLOC = -7
E_LAUNCH = -8
E_DEVICE_TIMEOUT = -9
E_ABI = -10
E_WORKSPACE = -11
E_SCRATCH_LIMIT = -12
NOALLOC_SCRATCH_BYTES = (4 << 20) + (64 << 10)

_u32, _u64, _f = C.c_uint32, C.c_uint64, C.c_float
_HDR = [("grid_dim", _u32 * 3), ("block_dim", _u32 * 3), ("M", _u32), ("N", _u32), ("K", _u32)]


class KbtSgemmArg(C.Structure):  # benchmarks/kbt_sgemm/common.h:4-13
    _fields_ = _HDR + [("a_addr", _u64), ("b_addr", _u64), ("c_addr", _u64)]


class KbtGemmAddReluArg(C.Structure):  # benchmarks/kbt_gemm_add_relu/common.h:4-14
    _fields_ = _HDR + [("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64), ("c_addr", _u64)]


class KbtGemmMulLeakyreluArg(C.Structure):  # benchmarks/kbt_gemm_mul_leakyrelu/common.h:4-16
    _fields_ = _HDR + [("multiplier", _f), ("negative_slope", _f), ("a_addr", _u64), ("w_addr", _u64),
                       ("bias_addr", _u64), ("c_addr", _u64)]


class KbtGemmDivSumScaleArg(C.Structure):  # benchmarks/kbt_gemm_div_sum_scale/common.h:4-14
    _fields_ = _HDR + [("scaling_factor", _f), ("a_addr", _u64), ("w_addr", _u64), ("c_addr", _u64)]


class KbtGemmLayernormArg(C.Structure):  # benchmarks/kbt_gemm_layernorm/common.h:4-17
    _fields_ = _HDR + [("eps", _f), ("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64),
                       ("ln_w_addr", _u64), ("ln_b_addr", _u64), ("c_addr", _u64)]


class KbtAttentionScoreArg(C.Structure):  # benchmarks/kbt_attention_score/common.h:4-13
    _fields_ = [("grid_dim", _u32 * 3), ("block_dim", _u32 * 3), ("M", _u32), ("N", _u32), ("D", _u32),
                ("q_addr", _u64), ("k_addr", _u64), ("c_addr", _u64)]


class KbtMatmulSoftmaxArg(C.Structure):  # benchmarks/kbt_matmul_softmax/common.h:4-13
    _fields_ = _HDR + [("a_addr", _u64), ("b_addr", _u64), ("c_addr", _u64)]


class KbtMatmulScaleResidaddClampArg(C.Structure):  # benchmarks/kbt_matmul_scale_residadd_clamp/common.h:4-17
    _fields_ = _HDR + [("scale_factor", _f), ("clamp_min", _f), ("clamp_max", _f), ("a_addr", _u64),
                       ("b_addr", _u64), ("c_addr", _u64), ("temp_addr", _u64)]


class KbtMatmulSumMaxAvgpoolArg(C.Structure):  # benchmarks/kbt_matmul_sum_max_avgpool/common.h:4-14
    _fields_ = _HDR + [("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64), ("c_addr", _u64)]


class KbtGemmRmsnormSwigluArg(C.Structure):  # benchmarks/kbt_gemm_rmsnorm_swiglu/common.h:4-18
    _fields_ = _HDR + [("eps", _f), ("x_addr", _u64), ("rms_w_addr", _u64), ("wg_addr", _u64),
                       ("wu_addr", _u64), ("norm_addr", _u64), ("gate_addr", _u64), ("c_addr", _u64)]


class KbtGemmSiluMulArg(C.Structure):  # benchmarks/kbt_gemm_silu_mul/common.h:4-17
    _fields_ = _HDR + [("a_addr", _u64), ("wa_addr", _u64), ("ba_addr", _u64), ("wb_addr", _u64),
                       ("bb_addr", _u64), ("gate_addr", _u64), ("c_addr", _u64)]


class FlashArg(C.Structure):  # benchmarks/flash/common.h:8-20
    _fields_ = [("grid_dim", _u32 * 1), ("block_dim", _u32 * 1), ("kernel_type", _u32), ("seq_len", _u32),
                ("head_dim", _u32), ("block_size_r", _u32), ("block_size_c", _u32), ("Q_addr", _u64),
                ("K_addr", _u64), ("V_addr", _u64), ("O_addr", _u64)]


class AkiliEx(C.Structure):  # include/akili.h akili_ex_t
    _fields_ = [("abi_version", _u32), ("in_dtype", _u32), ("out_dtype", _u32), ("batch", _u32),
                ("heads", _u32), ("softmax_scale", _f), ("causal", _u32), ("flags", _u32),
                ("workspace", _u64), ("workspace_bytes", _u64)]


class AttentionArg(C.Structure):  # benchmarks/attention/common.h:8-19
    _fields_ = [("grid_dim", _u32 * 2), ("N", _u32), ("d", _u32), ("Q_addr", _u64), ("K_addr", _u64),
                ("S_addr", _u64), ("P_addr", _u64), ("V_addr", _u64), ("O_addr", _u64), ("kernel_id", _u32)]


class MatmulKernelArgs(C.Structure):  # benchmarks/llama2/common.h:3-12
    _fields_ = [("grid_dim", _u32 * 2), ("block_dim", _u32 * 2), ("A_addr", _u64), ("B_addr", _u64),
                ("C_addr", _u64), ("M", C.c_int32), ("N", C.c_int32), ("K", C.c_int32)]


class MatvecSeg(C.Structure):  # include/akili.h akili_matvec_seg_t
    _fields_ = [("W_addr", _u64), ("C_addr", _u64), ("rows", C.c_int32), ("reserved", C.c_int32)]


# ---- kb2_* structs (benchmarks/kb2_<bench>/common.h): no launch fields ----
_MNK = [("M", _u32), ("N", _u32), ("K", _u32)]


class Kb2GemmAddReluArg(C.Structure):  # benchmarks/kb2_gemm_add_relu/common.h
    _fields_ = _MNK + [("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64), ("c_addr", _u64)]


class Kb2GemmMulLeakyreluArg(C.Structure):  # benchmarks/kb2_gemm_mul_leakyrelu/common.h
    _fields_ = _MNK + [("multiplier", _f), ("negative_slope", _f), ("a_addr", _u64), ("w_addr", _u64),
                       ("bias_addr", _u64), ("c_addr", _u64)]


class Kb2GemmDivSumScaleArg(C.Structure):  # benchmarks/kb2_gemm_div_sum_scale/common.h
    _fields_ = _MNK + [("scaling_factor", _f), ("a_addr", _u64), ("w_addr", _u64), ("c_addr", _u64)]


class Kb2GemmLayernormArg(C.Structure):  # benchmarks/kb2_gemm_layernorm/common.h
    _fields_ = _MNK + [("eps", _f), ("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64), ("ln_w_addr", _u64),
                       ("ln_b_addr", _u64), ("c_addr", _u64)]


class Kb2AttentionScoreArg(C.Structure):  # benchmarks/kb2_attention_score/common.h
    _fields_ = [("M", _u32), ("N", _u32), ("D", _u32), ("q_addr", _u64), ("k_addr", _u64), ("c_addr", _u64)]


class Kb2MatmulSoftmaxArg(C.Structure):  # benchmarks/kb2_matmul_softmax/common.h
    _fields_ = _MNK + [("a_addr", _u64), ("b_addr", _u64), ("c_addr", _u64)]


class Kb2MatmulScaleResidaddClampArg(C.Structure):  # benchmarks/kb2_matmul_scale_residadd_clamp/common.h
    _fields_ = _MNK + [("scale_factor", _f), ("clamp_min", _f), ("clamp_max", _f), ("a_addr", _u64),
                       ("w_addr", _u64), ("bias_addr", _u64), ("c_addr", _u64)]


class Kb2MatmulSumMaxAvgpoolArg(C.Structure):  # benchmarks/kb2_matmul_sum_max_avgpool/common.h
    _fields_ = _MNK + [("a_addr", _u64), ("w_addr", _u64), ("bias_addr", _u64), ("c_addr", _u64)]


class Kb2GemmRmsnormSwigluArg(C.Structure):  # benchmarks/kb2_gemm_rmsnorm_swiglu/common.h
    _fields_ = _MNK + [("eps", _f), ("x_addr", _u64), ("rms_w_addr", _u64), ("wg_addr", _u64), ("wu_addr", _u64),
                       ("c_addr", _u64)]


class Kb2GemmSiluMulArg(C.Structure):  # benchmarks/kb2_gemm_silu_mul/common.h
    _fields_ = _MNK + [("a_addr", _u64), ("wa_addr", _u64), ("ba_addr", _u64), ("wb_addr", _u64), ("bb_addr", _u64),
                       ("c_addr", _u64)]


# name -> (struct, buffer fields in harness upload order + outputs, sizeof in the reference)
OPS = {
    "kbt_sgemm": (KbtSgemmArg, 64),
    "kbt_gemm_add_relu": (KbtGemmAddReluArg, 72),
    "kbt_gemm_mul_leakyrelu": (KbtGemmMulLeakyreluArg, 80),
    "kbt_gemm_div_sum_scale": (KbtGemmDivSumScaleArg, 64),
    "kbt_gemm_layernorm": (KbtGemmLayernormArg, 88),
    "kbt_attention_score": (KbtAttentionScoreArg, 64),
    "kbt_matmul_softmax": (KbtMatmulSoftmaxArg, 64),
    "kbt_matmul_scale_residadd_clamp": (KbtMatmulScaleResidaddClampArg, 80),
    "kbt_matmul_sum_max_avgpool": (KbtMatmulSumMaxAvgpoolArg, 72),
    "kbt_gemm_rmsnorm_swiglu": (KbtGemmRmsnormSwigluArg, 96),
    "kbt_gemm_silu_mul": (KbtGemmSiluMulArg, 96),
    "flash": (FlashArg, 64),
    "kb2_gemm_add_relu": (Kb2GemmAddReluArg, 48),
    "kb2_gemm_mul_leakyrelu": (Kb2GemmMulLeakyreluArg, 56),
    "kb2_gemm_div_sum_scale": (Kb2GemmDivSumScaleArg, 40),
    "kb2_gemm_layernorm": (Kb2GemmLayernormArg, 64),
    "kb2_attention_score": (Kb2AttentionScoreArg, 40),
    "kb2_matmul_softmax": (Kb2MatmulSoftmaxArg, 40),
    "kb2_matmul_scale_residadd_clamp": (Kb2MatmulScaleResidaddClampArg, 56),
    "kb2_matmul_sum_max_avgpool": (Kb2MatmulSumMaxAvgpoolArg, 48),
    "kb2_gemm_rmsnorm_swiglu": (Kb2GemmRmsnormSwigluArg, 56),
    "kb2_gemm_silu_mul": (Kb2GemmSiluMulArg, 64),
}

_LIB = None


def load(path: str = LIB_PATH) -> C.CDLL:
    """Open libakili.so and declare its exports.  Raises if it is not built."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not os.path.exists(path):
        raise FileNotFoundError(
            f"{path} is not built; run `python -m akili_bench_b200.build` (the CUDA path has no fallback)")
    L = C.CDLL(path)
    for name, (st, _) in OPS.items():
        f = getattr(L, f"akili_{name}")
        f.argtypes = [C.POINTER(st), C.c_void_p]
        f.restype = C.c_int
        fx = getattr(L, f"akili_{name}_ex")
        fx.argtypes = [C.POINTER(st), C.POINTER(AkiliEx), C.c_void_p]
        fx.restype = C.c_int
    L.akili_attention.argtypes = [C.POINTER(AttentionArg), C.c_void_p]
    L.akili_attention.restype = C.c_int
    L.akili_attention_ex.argtypes = [C.POINTER(AttentionArg), C.POINTER(AkiliEx), C.c_void_p]
    L.akili_attention_ex.restype = C.c_int
    L.akili_host_call.argtypes = [C.c_char_p, C.c_void_p, C.POINTER(AkiliEx), C.c_void_p]
    L.akili_host_call.restype = C.c_int
    L.akili_llama2_matmul.argtypes = [C.POINTER(MatmulKernelArgs), C.c_void_p]
    L.akili_llama2_matmul.restype = C.c_int
    L.akili_llama2_matvec_batch.argtypes = [C.POINTER(MatvecSeg), C.c_int, C.c_uint64, C.c_int32, C.c_void_p]
    L.akili_llama2_matvec_batch.restype = C.c_int
    L.akili_flash_ml_ex.argtypes = [C.POINTER(FlashArg), C.POINTER(AkiliEx), C.c_uint64, C.c_uint64, C.c_void_p]
    L.akili_flash_ml_ex.restype = C.c_int
    L.akili_kbt_gemm_layernorm_noalloc.argtypes = [C.POINTER(KbtGemmLayernormArg), C.POINTER(AkiliEx), C.c_void_p]
    L.akili_kbt_gemm_layernorm_noalloc.restype = C.c_int
    L.akili_strerror.argtypes = [C.c_int]
    L.akili_strerror.restype = C.c_char_p
    L.akili_workspace_bytes.argtypes = [C.c_char_p, C.c_void_p, C.POINTER(AkiliEx), C.POINTER(C.c_uint64)]
    L.akili_workspace_bytes.restype = C.c_int
    L.akili_device_status.argtypes = [C.POINTER(C.c_uint32), C.c_int]
    L.akili_device_status.restype = C.c_int
    L.akili_selftest_wait_timeout.argtypes = [C.c_uint32, C.c_void_p]
    L.akili_selftest_wait_timeout.restype = C.c_int
    L.akili_launch_count.argtypes = []
    L.akili_launch_count.restype = C.c_uint64
    L.akili_sm_clock_read.argtypes = [C.POINTER(C.c_uint64), C.POINTER(C.c_uint64), C.c_int]
    L.akili_sm_clock_read.restype = C.c_int
    L.akili_abi_version.argtypes = []
    L.akili_abi_version.restype = C.c_uint32
    _LIB = L
    return L


def make_ex(in_dtype=DTYPE_F16, out_dtype=DTYPE_F16, batch=0, heads=0, softmax_scale=0.0,
            workspace=0, workspace_bytes=0, causal=0) -> AkiliEx:
    return AkiliEx(ABI_VERSION, in_dtype, out_dtype, batch, heads, softmax_scale, causal, 0, workspace,
                   workspace_bytes)


def strerror(code: int) -> str:
    return load().akili_strerror(code).decode()


class AkiliError(RuntimeError):
    def __init__(self, op: str, code: int):
        super().__init__(f"akili_{op} returned {code}: {strerror(code)}")
        self.code = code


def call(op: str, arg, ex: AkiliEx | None = None, stream: int = 0) -> int:
    """Call akili_<op>(arg, stream) or akili_<op>_ex(arg, ex, stream); return the status code."""
    L = load()
    if ex is None:
        return getattr(L, f"akili_{op}")(C.byref(arg), C.c_void_p(stream))
    return getattr(L, f"akili_{op}_ex")(C.byref(arg), C.byref(ex), C.c_void_p(stream))


def check(op: str, arg, ex: AkiliEx | None = None, stream: int = 0) -> None:
    rc = call(op, arg, ex, stream)
    if rc != OK:
        raise AkiliError(op, rc)
