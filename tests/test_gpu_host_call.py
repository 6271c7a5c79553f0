"""akili_host_call: the GEMM-family ops on HOST buffers, with the copies and
the fused GEMM pipelined over row chunks.  Each output row comes from the
same kernel as on the device path, so the results are compared with the
device-buffer call (identical up to one fp16 ulp where the chunk changes the
GEMM kernel) and with the oracle to the parity bar.  M values leave a ragged
last chunk and more chunks than buffer slots."""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import abi, ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu


def pinned(t, pin=True):
    t = t.contiguous().cpu()
    return t.pin_memory() if pin else t.clone()


@pytest.mark.parametrize("M,pin", [(1000, True), (8192, True), (264, False), (8, True)])
def test_add_relu_host_matches_device_call(oracle, M, pin):
    N, K = 512, 256
    g = torch.Generator(device="cuda").manual_seed(M)
    x = torch.randn((M, K), generator=g, device="cuda").half()
    w = (torch.randn((K, N), generator=g, device="cuda") * K ** -0.5).half()
    b = torch.randn((N,), generator=g, device="cuda") * 0.1
    dev = ops.kbt_gemm_add_relu(x, w, b).cpu()
    out = torch.empty((M, N), dtype=torch.float16, pin_memory=pin)
    got = ops.kbt_gemm_add_relu_host(pinned(x, pin), pinned(w, pin), pinned(b, pin), out=out)
    diff = (got.float() - dev.float()).abs()
    assert (diff <= 1e-3 * dev.float().abs() + 1e-6).all(), float(diff.max())
    ref = oracle.kbt_gemm_add_relu(x.float().cpu().numpy(), w.float().cpu().numpy(), b.cpu().numpy(), M, N, K)
    assert_parity(got.float().numpy(), ref, what="add_relu host call")


def _arg(st, M, N, K, **addrs):
    a = st()
    a.M, a.N = M, N
    if hasattr(a, "K"):
        a.K = K
    else:
        a.D = K
    for k, v in addrs.items():
        setattr(a, f"{k}_addr", v.data_ptr())
    return a


def test_layernorm_and_rowsum_host_calls_fp32(oracle):
    M, N, K = 520, 256, 128
    rng = np.random.default_rng(3)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32)).pin_memory()
    w = torch.from_numpy((rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5)).pin_memory()
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.1).pin_memory()
    g = torch.from_numpy(1 + rng.standard_normal(N, dtype=np.float32) * 0.02).pin_memory()
    beta = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.02).pin_memory()
    c = torch.zeros((M, N), dtype=torch.float32).pin_memory()
    arg = _arg(abi.KbtGemmLayernormArg, M, N, K, a=x, w=w, bias=b, ln_w=g, ln_b=beta, c=c)
    arg.eps = 1e-5
    ops.host_call("kbt_gemm_layernorm", arg, torch.float32, torch.float32)
    dev = ops.kbt_gemm_layernorm(x.cuda(), w.cuda(), b.cuda(), g.cuda(), beta.cuda(), 1e-5).cpu()
    assert torch.allclose(c, dev, rtol=1e-5, atol=1e-5)
    v = torch.zeros(M, dtype=torch.float32).pin_memory()
    arg = _arg(abi.KbtGemmDivSumScaleArg, M, N, K, a=x, w=w, c=v)
    arg.scaling_factor = 2.0
    ops.host_call("kbt_gemm_div_sum_scale", arg, torch.float32, torch.float32)
    ref = oracle.kbt_gemm_div_sum_scale(x.half().float().numpy(), w.half().float().numpy(), M, N, K, 2.0)
    assert_parity(v.numpy(), ref, rows=False, what="div_sum_scale host call")


def test_swiglu_and_kb2_host_calls(oracle):
    M, N, K = 384, 256, 128
    rng = np.random.default_rng(4)
    x = torch.from_numpy(rng.standard_normal((M, K), dtype=np.float32))
    rw = torch.from_numpy(1 + rng.standard_normal(K, dtype=np.float32) * 0.02)
    wg = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5)
    wu = torch.from_numpy(rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5)
    c = torch.zeros((M, N), dtype=torch.float16).pin_memory()
    xh, wgh, wuh, rwh = x.half().pin_memory(), wg.half().pin_memory(), wu.half().pin_memory(), rw.pin_memory()
    arg = _arg(abi.KbtGemmRmsnormSwigluArg, M, N, K, x=xh, rms_w=rwh, wg=wgh, wu=wuh, c=c)
    arg.eps = 1e-6
    ops.host_call("kbt_gemm_rmsnorm_swiglu", arg, torch.float16, torch.float16)
    dev = ops.kbt_gemm_rmsnorm_swiglu(xh.cuda(), rw.cuda(), wgh.cuda(), wuh.cuda(), 1e-6).cpu()
    assert ((c.float() - dev.float()).abs() <= 1e-3 * dev.float().abs() + 1e-5).all()
    # kb2: fp32 operands at fp32 accuracy (split precision)
    b = torch.from_numpy(rng.standard_normal(N, dtype=np.float32) * 0.1)
    out = torch.zeros((M, N), dtype=torch.float32).pin_memory()
    keep = (x.pin_memory(), wg.pin_memory(), b.pin_memory())
    a2 = abi.Kb2GemmAddReluArg(M, N, K, keep[0].data_ptr(), keep[1].data_ptr(), keep[2].data_ptr(), out.data_ptr())
    ops.host_call("kb2_gemm_add_relu", a2, torch.float32, torch.float32)
    ref = oracle.kb2_gemm_add_relu(x.numpy(), wg.numpy(), b.numpy(), M, N, K)
    assert np.abs(out.numpy() - ref).max() <= 1e-4 * np.abs(ref).max()


@pytest.mark.parametrize("B,H,S,D,causal", [(2, 5, 300, 64, False), (1, 12, 256, 128, True), (3, 1, 64, 32, False)])
def test_flash_host_call_matches_device_call(B, H, S, D, causal):
    """Flash on host tensors goes through in chunks of heads; each head runs
    the same kernel as on the device path, so O is identical."""
    g = torch.Generator(device="cuda").manual_seed(S + H)
    q, k, v = (torch.randn((B, H, S, D), generator=g, device="cuda").half() for _ in range(3))
    dev = ops.flash(q, k, v, softmax_scale=D ** -0.5, causal=causal).cpu()
    hq, hk, hv = (t.cpu().pin_memory() for t in (q, k, v))
    got = ops.flash(hq, hk, hv, softmax_scale=D ** -0.5, causal=causal)
    assert not got.is_cuda
    assert torch.equal(got, dev)


def test_flash_host_call_fp32_reference_semantics():
    """The plain fp32 form (one unscaled head, pageable buffers)."""
    S, D = 200, 16
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn((S, D), generator=g) for _ in range(3))
    dev = ops.flash(q.cuda(), k.cuda(), v.cuda()).cpu()
    got = ops.flash(q, k, v)
    assert torch.equal(got, dev)
