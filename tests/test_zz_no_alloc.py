"""akili_kbt_gemm_layernorm_noalloc: the allocation-free form of kbt_gemm_layernorm.

Some callers cannot call cudaMalloc: a serving process whose allocator has
already reserved the GPU's memory, or a plugin host whose execute callback
must not allocate because cudaMalloc/cudaFree would synchronise the device in
the middle of its stream work.  This entry point keeps its only scratch (the
LayerNorm row statistics) in a fixed device array inside the library.

The GPU test calls it through the C ABI twice in a row (the second call sees
the array holding the first call's contents) and checks each output against
the existing akili_kbt_gemm_layernorm_ex on the same inputs, and against the
CPU oracle (the reference's LayerNorm gold loop) on the same fp16-rounded
operands, within the parity tolerance the other tests use.  It also checks
that the device's free memory is the same before and after the second call.  This
file is named so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from akili_bench_b200 import abi
from akili_bench_b200.parity import assert_parity


def _arg(M, N, K, addrs=(0x1000, 0x2000, 0x3000, 0x4000, 0x5000, 0x6000)):
    a = abi.KbtGemmLayernormArg()
    a.M, a.N, a.K, a.eps = M, N, K, 1e-5
    a.a_addr, a.w_addr, a.bias_addr, a.ln_w_addr, a.ln_b_addr, a.c_addr = addrs
    return a


def _noalloc(arg, ex, stream=0):
    return abi.load().akili_kbt_gemm_layernorm_noalloc(C.byref(arg), C.byref(ex), C.c_void_p(stream))


def test_noalloc_rejects_what_it_cannot_hold_without_touching_the_gpu():
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16)
    # 16 * M * ceil(N/256) bytes of partials must fit the fixed array
    big = _arg(65536, 8192, 64)
    assert 16 * 65536 * 32 > abi.NOALLOC_SCRATCH_BYTES
    assert _noalloc(big, ex) == abi.E_SCRATCH_LIMIT
    assert "no-alloc scratch" in abi.strerror(abi.E_SCRATCH_LIMIT)
    # fp32 operands would need converted copies, which the fixed scratch does not hold
    assert _noalloc(_arg(64, 256, 64), abi.make_ex(abi.DTYPE_F32, abi.DTYPE_F16)) == abi.E_DTYPE
    ex_ws = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16, workspace=0x10000, workspace_bytes=1 << 20)
    assert _noalloc(_arg(64, 256, 64), ex_ws) == abi.E_UNSUPPORTED
    assert abi.load().akili_kbt_gemm_layernorm_noalloc(C.byref(_arg(64, 256, 64)), None, None) == abi.E_NULL_ARG
    # the documented example fits: 4 MiB of statistics plus 512 bytes of counters at M = 16384, N = 4096
    # (checked only where no GPU would go on to launch on these placeholder addresses)
    try:
        import torch
        have_gpu = torch.cuda.is_available()
    except Exception:
        have_gpu = False
    if not have_gpu:
        assert 16 * 16384 * 16 + 512 <= abi.NOALLOC_SCRATCH_BYTES
        assert _noalloc(_arg(16384, 4096, 64), ex) not in (abi.OK, abi.E_SCRATCH_LIMIT)  # no device here
        assert _noalloc(_arg(16384, 4608, 64), ex) == abi.E_SCRATCH_LIMIT


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K,out_dtype", [(200, 4096, 256, "f16"), (136, 1048, 72, "f32")])
def test_noalloc_matches_existing_entry_on_two_calls_in_a_row(oracle, M, N, K, out_dtype):
    torch = pytest.importorskip("torch")
    from akili_bench_b200 import ops
    rng = np.random.default_rng(M + N)
    f16, f32 = torch.float16, torch.float32
    odt = f16 if out_dtype == "f16" else f32
    odt_code = abi.DTYPE_F16 if out_dtype == "f16" else abi.DTYPE_F32
    for call in range(2):
        x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).cuda().to(f16)
        w = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5).cuda().to(f16)
        b = torch.from_numpy(rng.standard_normal(N).astype(np.float32) * 0.02).cuda()
        g = torch.from_numpy((1 + rng.standard_normal(N) * 0.02).astype(np.float32)).cuda()
        beta = torch.from_numpy(rng.standard_normal(N).astype(np.float32) * 0.02).cuda()
        ref = ops.kbt_gemm_layernorm(x, w, b, g, beta, 1e-5, out_dtype=odt)
        out = torch.full((M, N), float("nan"), device="cuda", dtype=odt)
        arg = _arg(M, N, K, (x.data_ptr(), w.data_ptr(), b.data_ptr(), g.data_ptr(), beta.data_ptr(),
                             out.data_ptr()))
        torch.cuda.synchronize()
        free_before = torch.cuda.mem_get_info()[0]
        rc = _noalloc(arg, abi.make_ex(abi.DTYPE_F16, odt_code), torch.cuda.current_stream().cuda_stream)
        assert rc == abi.OK, abi.strerror(rc)
        torch.cuda.synchronize()
        if call:  # (the first call on a device may still load kernel code lazily and resolves the array's address)
            assert torch.cuda.mem_get_info()[0] == free_before  # nothing was allocated on the device
        assert ops.device_status() == 0
        got = out.float().cpu().numpy()
        assert_parity(got, ref.float().cpu().numpy(), what=f"noalloc call {call} vs akili_kbt_gemm_layernorm_ex")
        gold = oracle.kbt_gemm_layernorm(x.float().cpu().numpy(), w.float().cpu().numpy(), b.cpu().numpy(),
                                         g.cpu().numpy(), beta.cpu().numpy(), M, N, K, 1e-5, threads=8)
        assert_parity(got, gold, what=f"noalloc call {call} vs oracle")
