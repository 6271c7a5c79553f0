"""Stream-K mode of the CTA-pair GEMM kernel, against the oracle and the
whole-tile mode.

When a GEMM's 256-row tiles fill the CTA pairs' waves poorly (the small
per-GPU M of a row-split GEMM: C2's 8192 rows over 8 GPUs leave 64 tiles for
74 pairs), the (tile, K-block) units are split evenly over the pairs; a
tile's owner adds the partial accumulators of the pairs that computed its
earlier K-blocks before the epilogue.  AKILI_STREAMK=1 selects it (whole
tiles are the default).
Each case checks the stream-K output against the oracle on sampled rows
(the parity bar) and against the whole-tile output on every element (the
two differ only in the order of the fp32 K-block sums), and the launch
count.  Shapes cover ragged M, N and K, the dual GEMM, a row-sum epilogue,
the log-sum-exp epilogue and the split (fp32) mode.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu


def f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float16).astype(np.float32)


def dev(x, dtype=torch.float16):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def sample_rows(M):
    return sorted({0, 1, 127, 128, 255, 256, M // 2, M - 129, M - 2, M - 1} & set(range(M)))


def both_modes(monkeypatch, run):
    """run() -> tensor, under stream-K and whole tiles; returns both as numpy."""
    outs = []
    for mode in ("1", "0"):
        monkeypatch.setenv("AKILI_STREAMK", mode)
        torch.cuda.synchronize()
        out = run().float().cpu().numpy()
        assert ops.device_status() == 0
        outs.append(out)
    return outs


def close(a, b, rtol=2e-3):
    """Stream-K against whole tiles: fp16 outputs may round the other way."""
    scale = np.abs(b).max() + 1e-30
    assert np.abs(a - b).max() <= rtol * scale


@pytest.mark.parametrize("M,N,K", [(1024, 4096, 4096), (2048, 1024, 2048), (1024, 1024, 4096), (264, 1040, 4104),
                                   (1000, 1000, 1032)])
def test_streamk_add_relu(oracle, monkeypatch, M, N, K):
    rng = np.random.default_rng(M + 3 * N + K)
    x, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_gemm_add_relu(dev(x), dev(w), dev(b, torch.float32),
                                                                   out_dtype=torch.float32))
    close(sk, dp, 1e-5)
    rows = sample_rows(M)
    ref = oracle.kbt_gemm_add_relu(np.ascontiguousarray(x[rows]), w, b, len(rows), N, K, threads=8)
    assert_parity(sk[rows], ref, what="add_relu stream-K")


def test_streamk_and_whole_tiles_are_one_launch(monkeypatch):
    """1024 rows at C2's N and K take stream-K (64 tiles for 74 pairs), 8192 rows whole tiles (6.9 waves)."""
    rng = np.random.default_rng(5)
    monkeypatch.setenv("AKILI_STREAMK", "1")
    for M in (1024, 8192):
        x, w = f16(rng, (M, 4096)), f16(rng, (4096, 4096), 4096 ** -0.5)
        b = np.zeros(4096, np.float32)
        xd, wd, bd = dev(x), dev(w), dev(b, torch.float32)
        ops.kbt_gemm_add_relu(xd, wd, bd)
        torch.cuda.synchronize()
        l0 = ops.launch_count()
        ops.kbt_gemm_add_relu(xd, wd, bd)
        torch.cuda.synchronize()
        assert ops.launch_count() - l0 == 1
    assert ops.device_status() == 0


@pytest.mark.parametrize("M,N,K", [(1032, 1000, 2048), (2048, 2048, 1024)])
def test_streamk_silu_mul_dual(oracle, monkeypatch, M, N, K):
    rng = np.random.default_rng(M * 5 + N)
    a, wa, wb = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5), f16(rng, (K, N), K ** -0.5)
    ba, bb = (rng.standard_normal(N).astype(np.float32) * 0.02 for _ in range(2))
    f32 = torch.float32
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_gemm_silu_mul(dev(a), dev(wa), dev(ba, f32), dev(wb),
                                                                   dev(bb, f32), out_dtype=f32))
    close(sk, dp, 1e-5)
    rows = sample_rows(M)
    ref = oracle.kbt_gemm_silu_mul(np.ascontiguousarray(a[rows]), wa, ba, wb, bb, len(rows), N, K, threads=8)
    assert_parity(sk[rows], ref, what="silu_mul stream-K")


def test_streamk_rmsnorm_swiglu_fp16(oracle, monkeypatch):
    M, N, K = 1024, 2048, 2048
    rng = np.random.default_rng(77)
    x = f16(rng, (M, K))
    rw = (1 + rng.standard_normal(K) * 0.02).astype(np.float32)
    wg, wu = f16(rng, (K, N), K ** -0.5), f16(rng, (K, N), K ** -0.5)
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_gemm_rmsnorm_swiglu(dev(x), dev(rw, torch.float32), dev(wg),
                                                                         dev(wu), 1e-6))
    close(sk, dp)
    rows = sample_rows(M)
    ref = oracle.kbt_gemm_rmsnorm_swiglu(np.ascontiguousarray(x[rows]), rw, wg, wu, len(rows), N, K, 1e-6,
                                         threads=8)
    assert_parity(sk[rows], ref, what="rmsnorm_swiglu stream-K")


def test_streamk_row_sums_and_lse(oracle, monkeypatch):
    M, N, K = 1024, 2048, 2048
    rng = np.random.default_rng(91)
    a, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    rows = sample_rows(M)
    ar = np.ascontiguousarray(a[rows])
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_gemm_div_sum_scale(dev(a), dev(w), 2.0, out_dtype=torch.float32))
    close(sk, dp, 1e-4)
    assert_parity(sk[rows], oracle.kbt_gemm_div_sum_scale(ar, w, len(rows), N, K, 2.0, threads=8), rows=False,
                  what="div_sum_scale stream-K")
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_matmul_sum_max_avgpool(dev(a), dev(w), dev(b, torch.float32),
                                                                            out_dtype=torch.float32))
    close(sk, dp, 1e-4)
    sk, dp = both_modes(monkeypatch, lambda: ops.kbt_matmul_scale_residadd_clamp(dev(a), dev(w), 0.5, -2.0, 2.0,
                                                                                 out_dtype=torch.float32))
    close(sk, dp, 1e-5)
    assert_parity(sk[rows], oracle.kbt_matmul_scale_residadd_clamp(ar, w, len(rows), N, K, 0.5, -2.0, 2.0,
                                                                   threads=8), rows=False, what="clamp stream-K")


def test_streamk_kb2_split_mode(oracle, monkeypatch):
    """fp32 operands as fp16 hi + lo parts (three MMAs per K-step) under stream-K."""
    M, N, K = 1024, 1024, 4096
    rng = np.random.default_rng(31)
    x = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((K, N), dtype=np.float32) * K ** -0.5
    b = rng.standard_normal(N).astype(np.float32) * 0.1
    f32 = torch.float32
    sk, dp = both_modes(monkeypatch, lambda: ops.kb2_gemm_add_relu(dev(x, f32), dev(w, f32), dev(b, f32)))
    close(sk, dp, 1e-4)  # the split mode's own bar (about 2^-21 per product)
    rows = sample_rows(M)
    ref = oracle.kb2_gemm_add_relu(np.ascontiguousarray(x[rows]), w, b, len(rows), N, K, threads=8)
    scale = np.abs(ref).max()
    assert np.abs(sk[rows] - ref).max() <= 1e-4 * scale
