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
