"""GPU parity of akili_attention (benchmarks/attention: the unfused
three-kernel attention on fp32 buffers) against the oracle's restatement of
its matmul_cpu / softmax_cpu.  The products keep the reference's summation
order, so S and O are compared bit for bit; the softmax within 1e-6 relative.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import abi  # noqa: E402

pytestmark = pytest.mark.gpu


def _run(kernel_id, N, d, **bufs):
    t = {k: torch.from_numpy(np.ascontiguousarray(v, dtype=np.float32)).cuda() for k, v in bufs.items()}
    out_name, shape = {0: ("S", (N, N)), 1: ("P", (N, N)), 2: ("O", (N, d))}[kernel_id]
    t[out_name] = torch.zeros(shape, device="cuda", dtype=torch.float32)
    arg = abi.AttentionArg()
    arg.N, arg.d, arg.kernel_id = N, d, kernel_id
    for k, v in t.items():
        setattr(arg, f"{k}_addr", v.data_ptr())
    rc = abi.load().akili_attention(arg, None)
    assert rc == abi.OK, abi.strerror(rc)
    torch.cuda.synchronize()
    return t[out_name].cpu().numpy()


@pytest.mark.parametrize("N,d", [(64, 8), (200, 24), (256, 32), (1000, 64)])
def test_three_kernels(oracle, N, d):
    rng = np.random.default_rng(N + d)
    q = (rng.random((N, d), dtype=np.float32) * 10 - 5)
    k = (rng.random((d, N), dtype=np.float32) * 10 - 5)  # K stored d x N, as the reference does
    v = (rng.random((N, d), dtype=np.float32) * 10 - 5)
    s = _run(0, N, d, Q=q, K=k)
    assert np.array_equal(s, oracle.attention_matmul(q, k, N, N, d))
    p = _run(1, N, d, S=s)
    ref_p = oracle.attention_softmax(s, N, N)
    np.testing.assert_allclose(p, ref_p, rtol=1e-6, atol=1e-9)
    o = _run(2, N, d, P=p, V=v)
    assert np.array_equal(o, oracle.attention_matmul(p, v, N, d, N))


def test_validation():
    arg = abi.AttentionArg()
    arg.N, arg.d, arg.kernel_id = 64, 8, 3
    arg.Q_addr = arg.K_addr = arg.S_addr = arg.P_addr = arg.V_addr = arg.O_addr = 0x1000
    assert abi.load().akili_attention(arg, None) == abi.E_UNSUPPORTED
    arg.kernel_id, arg.S_addr = 0, 0
    assert abi.load().akili_attention(arg, None) == abi.E_NULL_ARG


# ---- akili_attention_ex: batched heads, softmax scale, fp16 on the tensor cores ----

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402


def _torch_ref(q, k_t, v, scale):
    s = torch.matmul(q.float(), k_t.float())
    p = torch.softmax(s * scale, dim=-1)
    return torch.matmul(p, v.float()), s, p


@pytest.mark.parametrize("B,H,N,d", [(1, 3, 64, 64), (2, 2, 200, 128), (1, 2, 256, 32), (1, 1, 1024, 128)])
def test_attention_ex_fp16_tensor_cores(B, H, N, d):
    """fp16 Q/K/V; S and O from the tensor-core GEMM (fp32 accumulation,
    fp16 results), P from the one-pass softmax.  Against an fp32 reference of
    the same fp16 operands: S within fp16 rounding, P's rows sum to 1, and O
    to the parity bar (max|err| <= 1e-2 max|ref|, row cosine >= 0.9999)."""
    g = torch.Generator(device="cuda").manual_seed(N + d)
    q = torch.randn((B, H, N, d), generator=g, device="cuda").half()
    k_t = torch.randn((B, H, d, N), generator=g, device="cuda").half()
    v = torch.randn((B, H, N, d), generator=g, device="cuda").half()
    scale = d ** -0.5
    o, s, p = ops.attention_unfused(q, k_t, v, softmax_scale=scale)
    torch.cuda.synchronize()
    ref_o, ref_s, ref_p = _torch_ref(q, k_t, v, scale)
    assert (s.float() - ref_s).abs().max().item() <= 2e-3 * ref_s.abs().max().item()
    assert (p.float().sum(-1) - 1).abs().max().item() < 5e-3
    assert (p.float() - ref_p).abs().max().item() < 2e-3
    assert_parity(o.float().reshape(-1, d).cpu().numpy(), ref_o.reshape(-1, d).cpu().numpy(), what="attention fp16")


def test_attention_ex_fp32_batched_matches_oracle(oracle):
    """fp32 heads through the _ex form: each head bit-identical to the exact
    kernels' S and O, the softmax with a scale."""
    B, H, N, d = 1, 3, 96, 16
    rng = np.random.default_rng(7)
    q = rng.random((B, H, N, d), dtype=np.float32) * 4 - 2
    k_t = rng.random((B, H, d, N), dtype=np.float32) * 4 - 2
    v = rng.random((B, H, N, d), dtype=np.float32) * 4 - 2
    o, s, p = ops.attention_unfused(*(torch.from_numpy(x).cuda() for x in (q, k_t, v)), softmax_scale=0.25)
    torch.cuda.synchronize()
    s, p, o = s.cpu().numpy(), p.cpu().numpy(), o.cpu().numpy()
    for h in range(H):
        assert np.array_equal(s[0, h], oracle.attention_matmul(q[0, h], k_t[0, h], N, N, d))
        ref_p = oracle.attention_softmax(np.ascontiguousarray(s[0, h] * np.float32(0.25)), N, N)
        np.testing.assert_allclose(p[0, h], ref_p, rtol=1e-5, atol=1e-8)
        assert np.array_equal(o[0, h], oracle.attention_matmul(p[0, h], v[0, h], N, d, N))


def test_attention_ex_validation():
    arg = abi.AttentionArg()
    arg.N, arg.d, arg.kernel_id = 64, 12, 0
    arg.Q_addr = arg.K_addr = arg.S_addr = arg.P_addr = arg.V_addr = arg.O_addr = 0x1000
    L = abi.load()
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16, batch=1, heads=2)
    assert L.akili_attention_ex(arg, ex, None) == abi.E_SHAPE          # d % 8 on the fp16 path
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F32)
    assert L.akili_attention_ex(arg, ex, None) == abi.E_DTYPE          # mixed dtypes
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16, causal=1)
    assert L.akili_attention_ex(arg, ex, None) == abi.E_UNSUPPORTED
    assert L.akili_attention_ex(arg, None, None) == abi.E_NULL_ARG
