"""The C ABI without a GPU: the libraries load, export every declared symbol,
keep the reference struct layouts, and reject bad argument blocks with the
documented codes before touching CUDA."""
import ctypes as C
import os
import re
import subprocess

import pytest

from akili_bench_b200 import abi

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared(header: str, prefix: str) -> set[str]:
    text = open(os.path.join(ROOT, "include", header)).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return set(re.findall(rf"\b({prefix}\w*)\s*\(", text))


def exported(lib: str) -> set[str]:
    out = subprocess.run(["nm", "-D", "--defined-only", lib], capture_output=True, text=True, check=True).stdout
    return {ln.split()[-1] for ln in out.splitlines() if " T " in ln}


def test_libakili_exports_every_declared_entry():
    names = declared("akili.h", "akili_")
    # kbt+flash, kb2, attention (+ex), flash statistics, no-alloc LN, llama2 matmul + batch, helpers
    assert len(names) == 24 + 20 + 2 + 1 + 1 + 2 + 8  # helpers: + akili_host_call, akili_sm_clock_read
    missing = names - exported(abi.LIB_PATH)
    assert not missing, missing
    L = abi.load()
    for n in names:
        assert getattr(L, n) is not None


def test_vortex_shim_exports_the_runtime_api():
    names = declared("vortex.h", "vx_")
    assert {"vx_start", "vx_ready_wait", "vx_mem_alloc", "vx_upload_bytes"} <= names
    missing = names - exported(abi.VORTEX_LIB_PATH)
    assert not missing, missing
    C.CDLL(abi.VORTEX_LIB_PATH)


def test_header_static_asserts_compile_and_match_ctypes():
    r = subprocess.run(["g++", "-std=c++17", "-fsyntax-only", "-x", "c++", os.path.join(ROOT, "include", "akili.h")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    for name, (st, size) in abi.OPS.items():
        assert C.sizeof(st) == size, name
    assert C.sizeof(abi.AkiliEx) == 48
    assert abi.KbtGemmLayernormArg.c_addr.offset == 80
    assert abi.KbtMatmulScaleResidaddClampArg.temp_addr.offset == 72
    assert abi.FlashArg.Q_addr.offset == 32 and abi.FlashArg.block_size_c.offset == 24


def test_abi_version_and_strerror():
    L = abi.load()
    assert L.akili_abi_version() == abi.ABI_VERSION
    for code in range(0, -13, -1):
        assert abi.strerror(code) != "unknown error"
    assert abi.strerror(-99) == "unknown error"


def _valid_add_relu():
    a = abi.KbtGemmAddReluArg()
    a.M, a.N, a.K = 64, 64, 64
    a.a_addr, a.w_addr, a.bias_addr, a.c_addr = 0x10000, 0x20000, 0x30000, 0x40000
    return a


def test_validation_codes_before_any_cuda_call():
    L = abi.load()
    assert L.akili_kbt_gemm_add_relu(None, None) == abi.E_NULL_ARG
    a = _valid_add_relu()
    a.M = 12
    assert abi.call("kbt_gemm_add_relu", a) == abi.E_SHAPE
    a = _valid_add_relu()
    a.K = 0
    assert abi.call("kbt_gemm_add_relu", a) == abi.E_SHAPE
    a = _valid_add_relu()
    a.bias_addr = 0
    assert abi.call("kbt_gemm_add_relu", a) == abi.E_NULL_ARG
    a = _valid_add_relu()
    a.w_addr += 4
    assert abi.call("kbt_gemm_add_relu", a) == abi.E_ALIGN
    ex = abi.make_ex()
    ex.abi_version = 99
    assert abi.call("kbt_gemm_add_relu", _valid_add_relu(), ex) == abi.E_ABI
    ex = abi.make_ex(in_dtype=7)
    assert abi.call("kbt_gemm_add_relu", _valid_add_relu(), ex) == abi.E_DTYPE
    ex = abi.make_ex()
    ex.causal = 1
    assert abi.call("kbt_gemm_add_relu", _valid_add_relu(), ex) == abi.E_UNSUPPORTED
    assert L.akili_kbt_gemm_add_relu_ex(C.byref(_valid_add_relu()), None, None) == abi.E_NULL_ARG
    f = abi.FlashArg()
    f.seq_len, f.head_dim = 64, 256
    f.Q_addr, f.K_addr, f.V_addr, f.O_addr = 0x1000, 0x2000, 0x3000, 0x4000
    assert abi.call("flash", f) == abi.E_UNSUPPORTED
    f.head_dim = 12
    assert abi.call("flash", f) == abi.E_SHAPE
    # causal is a flash option (0 or 1); the statistics entry needs both buffers
    f.head_dim = 64
    ex = abi.make_ex(causal=2)
    assert abi.call("flash", f, ex) == abi.E_UNSUPPORTED
    ex = abi.make_ex(causal=1)
    assert L.akili_flash_ml_ex(C.byref(f), C.byref(ex), 0, 0x5000, None) == abi.E_NULL_ARG
    assert L.akili_flash_ml_ex(C.byref(f), C.byref(ex), 0x5002, 0x6000, None) == abi.E_ALIGN


def test_valid_args_without_a_gpu_report_no_device():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except ImportError:
        pass
    assert abi.call("kbt_gemm_add_relu", _valid_add_relu()) == abi.E_NO_DEVICE


def test_workspace_query_needs_no_buffers():
    L = abi.load()
    a = abi.KbtGemmLayernormArg()
    a.M, a.N, a.K = 16384, 4096, 4096
    n = C.c_uint64(0)
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16)
    assert L.akili_workspace_bytes(b"kbt_gemm_layernorm", C.byref(a), C.byref(ex), C.byref(n)) == 0
    assert n.value >= 2 * 16 * 16384 * 4  # (mean, M2) per row per 256-column tile
    assert L.akili_workspace_bytes(b"kbt_gemm_layernorm", C.byref(a), None, C.byref(n)) == 0
    assert n.value >= (16384 * 4096 + 4096 * 4096) * 2  # fp16 copies of the fp32 operands
    assert L.akili_workspace_bytes(b"nope", C.byref(a), None, C.byref(n)) == abi.E_UNSUPPORTED


def test_attention_ex_rejects_bad_modes_before_cuda():
    L = abi.load()
    arg = abi.AttentionArg()
    arg.N, arg.d, arg.kernel_id = 64, 16, 0
    arg.Q_addr = arg.K_addr = arg.S_addr = arg.P_addr = arg.V_addr = arg.O_addr = 0x1000
    assert L.akili_attention_ex(C.byref(arg), None, None) == abi.E_NULL_ARG
    assert L.akili_attention_ex(C.byref(arg), C.byref(abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F32)), None) == abi.E_DTYPE
    assert L.akili_attention_ex(C.byref(arg), C.byref(abi.make_ex(causal=1)), None) == abi.E_UNSUPPORTED
    arg.kernel_id = 3
    assert L.akili_attention_ex(C.byref(arg), C.byref(abi.make_ex()), None) == abi.E_UNSUPPORTED


def test_host_call_validates_before_cuda():
    L = abi.load()
    arg = abi.KbtGemmAddReluArg()
    arg.M, arg.N, arg.K = 64, 64, 64
    assert L.akili_host_call(b"no_such_op", C.byref(arg), None, None) == abi.E_UNSUPPORTED
    assert L.akili_host_call(None, C.byref(arg), None, None) == abi.E_NULL_ARG
    assert L.akili_host_call(b"kbt_gemm_add_relu", C.byref(arg), None, None) == abi.E_NULL_ARG  # host pointers 0
    arg.N = 60
    assert L.akili_host_call(b"kbt_gemm_add_relu", C.byref(arg), None, None) == abi.E_SHAPE
    k2 = abi.Kb2GemmAddReluArg(64, 64, 64, 0, 0, 0, 0)
    assert L.akili_host_call(b"kb2_gemm_add_relu", C.byref(k2), C.byref(abi.make_ex()), None) == abi.E_DTYPE
    assert L.akili_host_call(b"kbt_gemm_add_relu", C.byref(arg), C.byref(abi.make_ex(batch=2)), None) == \
        abi.E_UNSUPPORTED


def test_sm_clock_read_validates_before_any_cuda_call():
    L = abi.load()
    v = C.c_uint64(0)
    assert L.akili_sm_clock_read(None, C.byref(v), 0) == abi.E_NULL_ARG
    assert L.akili_sm_clock_read(C.byref(v), None, 0) == abi.E_NULL_ARG
