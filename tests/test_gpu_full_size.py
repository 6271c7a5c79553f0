"""Parity at the full configured sizes (add_relu x[8192,4096]·W[4096,4096];
layernorm x[16384,4096]; rmsnorm_swiglu x[16384,4096]·Wg/Wu[4096,11008];
flash B8 H32 S4096 d128), with the configured input distributions.

Every output is checked against properties that hold at any size.  Sampled
rows are also checked against the oracle, to the parity bar
(max|err| <= 1e-2 * max|ref|, row cosine >= 0.9999), on the same
fp16-rounded operands.  Rows are independent for every op, so the oracle
runs on the sampled rows alone.  The samples include the rows either side of
a CTA (128 rows) and a CTA-pair tile (256 rows) boundary, and the last rows.

The column tiles are never ragged at these shapes (4096 = 16 x 256 and
11008 = 43 x 256): the ragged-N paths (the TMA store clipping the last tile,
partial statistics slots) are covered in test_gpu_kbt.py, e.g. N = 4104,
8200 and 18952.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu


def rows_of(M):
    return sorted({0, 1, 127, 128, 255, 256, M // 3, M // 2, (2 * M) // 3, M - 129, M - 128, M - 2, M - 1})


def gen(seed):
    return torch.Generator(device="cuda").manual_seed(seed)


def randn(g, shape, std=1.0, mean=0.0, dtype=torch.float16):
    return (torch.randn(shape, generator=g, device="cuda") * std + mean).to(dtype)


def host(t):
    return np.ascontiguousarray(t.float().cpu().numpy())


def test_add_relu_c2(oracle):
    M, N, K = 8192, 4096, 4096
    g = gen(1)
    x, w = randn(g, (M, K)), randn(g, (K, N), K ** -0.5)
    b = randn(g, (N,), 0.1, dtype=torch.float32)
    out = ops.kbt_gemm_add_relu(x, w, b)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and (out >= 0).all()  # ReLU
    assert (out > 0).float().mean().item() > 0.3
    r = rows_of(M)
    ref = oracle.kbt_gemm_add_relu(host(x[r]), host(w), host(b), len(r), N, K, threads=8)
    assert_parity(host(out[r]), ref, what="add_relu C2")


def test_layernorm_c3(oracle):
    M, N, K = 16384, 4096, 4096
    g = gen(2)
    x, w = randn(g, (M, K)), randn(g, (K, N), K ** -0.5)
    b = randn(g, (N,), 0.02, dtype=torch.float32)
    gam, bet = randn(g, (N,), 0.02, 1.0, torch.float32), randn(g, (N,), 0.02, dtype=torch.float32)
    out = ops.kbt_gemm_layernorm(x, w, b, gam, bet, 1e-5)
    torch.cuda.synchronize()
    # every row, normalised back through the affine: mean 0 and variance 1
    z = (out.float() - bet) / gam
    assert z.mean(dim=1).abs().max().item() < 1e-2
    assert (z.var(dim=1, unbiased=False) - 1).abs().max().item() < 2e-2
    r = rows_of(M)
    ref = oracle.kbt_gemm_layernorm(host(x[r]), host(w), host(b), host(gam), host(bet), len(r), N, K, 1e-5,
                                    threads=8)
    assert_parity(host(out[r]), ref, what="layernorm C3")


def test_rmsnorm_swiglu_c4(oracle):
    M, N, K = 16384, 11008, 4096
    g = gen(3)
    x = randn(g, (M, K))
    rw = randn(g, (K,), 0.02, 1.0, torch.float32)
    wg, wu = randn(g, (K, N), K ** -0.5), randn(g, (K, N), K ** -0.5)
    out = ops.kbt_gemm_rmsnorm_swiglu(x, rw, wg, wu, 1e-6)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all()
    r = rows_of(M)
    ref = oracle.kbt_gemm_rmsnorm_swiglu(host(x[r]), host(rw), host(wg), host(wu), len(r), N, K, 1e-6, threads=8)
    assert_parity(host(out[r]), ref, what="rmsnorm_swiglu C4")


def test_matmul_softmax_c2_row_fused(oracle):
    """kbt_matmul_softmax at the C2 shape: the row-fused epilogue (row
    statistics merged across the 16 tiles of each row) in one launch."""
    M, N, K = 8192, 4096, 4096
    g = gen(5)
    a, b = randn(g, (M, K)), randn(g, (K, N), 3 * K ** -0.5)
    out = ops.kbt_matmul_softmax(a, b)
    torch.cuda.synchronize()
    assert torch.isfinite(out).all() and (out >= 0).all()
    assert (out.float().sum(dim=1) - 1).abs().max().item() < 5e-3  # every row sums to one
    r = rows_of(M)
    ref = oracle.kbt_matmul_softmax(host(a[r]), host(b), len(r), N, K, threads=8)
    assert_parity(host(out[r]), ref, what="matmul_softmax C2")


def test_flash_c5(oracle):
    B, H, S, D = 8, 32, 4096, 128
    g = gen(4)
    q, k, v = (randn(g, (B, H, S, D)) for _ in range(3))
    out = ops.flash(q, k, v, softmax_scale=D ** -0.5)
    torch.cuda.synchronize()
    # each output is a convex combination of V's rows, per head and column
    vmin, vmax = v.float().amin(dim=2, keepdim=True), v.float().amax(dim=2, keepdim=True)
    o = out.float()
    assert ((o >= vmin - 1e-2) & (o <= vmax + 1e-2)).all()
    r = rows_of(S)
    for b, h in [(0, 0), (3, 17), (7, 31)]:
        qh, kh, vh = host(q[b, h]), host(k[b, h]), host(v[b, h])
        ref = np.stack([oracle.flash(qh, kh, vh, S, D, D ** -0.5, i, i + 1)[i] for i in r])
        assert_parity(host(out[b, h])[r], ref, what=f"flash C5 head ({b}, {h})")
