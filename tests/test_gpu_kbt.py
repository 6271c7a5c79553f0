"""GPU parity of every kbt_* op against the CPU oracle, through the C ABI.

Inputs are seeded and rounded to fp16 once, so the oracle and the device see
identical operands.  Each op runs through both forms of its entry point:
akili_<bench> (fp32 buffers, reference semantics) and akili_<bench>_ex
(fp16 operands, fp16 output).  Shapes cover one tile, ragged M/N/K (not
multiples of the 128x256x64 tile, only of 8, as the reference harness
guarantees) and multi-tile rows for the full-row epilogues.
Tolerance: max|err| <= 1e-2 * max|ref| and per-row cosine >= 0.9999.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu

# M <= 128 runs the single-CTA kernel, larger M the CTA-pair kernel (256-row tiles).
SHAPES = [(16, 16, 16), (24, 40, 56), (128, 256, 64), (200, 264, 136), (136, 520, 1032), (392, 776, 200),
          (1000, 264, 72)]
ROW_SHAPES = [(16, 16, 16), (72, 1048, 200), (40, 4096, 128), (264, 4104, 136)]  # full-row epilogues, many tiles


def f16(rng, shape, scale=1.0, loc=0.0):
    return (rng.standard_normal(shape, dtype=np.float32) * scale + loc).astype(np.float16).astype(np.float32)


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


def both_forms(run, ref, rows=True, what=""):
    """run(dtype) -> torch output; checks fp32 (plain ABI) and fp16 (_ex ABI)."""
    for dt in (torch.float32, torch.float16):
        got = run(dt).float().cpu().numpy()
        torch.cuda.synchronize()
        assert ops.device_status() == 0
        assert_parity(got, ref, rows=rows, what=f"{what} {dt}")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kbt_sgemm(oracle, M, N, K):
    rng = np.random.default_rng(M * 7 + N)
    a, b = f16(rng, (M, K)), f16(rng, (K, N))
    ref = oracle.kbt_sgemm(a, b, M, N, K)
    both_forms(lambda dt: ops.kbt_sgemm(dev(a, dt), dev(b, dt), out_dtype=dt), ref, what="sgemm")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kbt_gemm_add_relu(oracle, M, N, K):
    rng = np.random.default_rng(M + N + K)
    x, w, b = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5), rng.standard_normal(N).astype(np.float32) * 0.1
    ref = oracle.kbt_gemm_add_relu(x, w, b, M, N, K)
    both_forms(lambda dt: ops.kbt_gemm_add_relu(dev(x, dt), dev(w, dt), dev(b, torch.float32), out_dtype=dt), ref,
               what="add_relu")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kbt_gemm_mul_leakyrelu(oracle, M, N, K):
    rng = np.random.default_rng(3 * M + N)
    x, w, b = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5), rng.standard_normal(N).astype(np.float32) * 0.1
    ref = oracle.kbt_gemm_mul_leakyrelu(x, w, b, M, N, K, 1.5, 0.01)
    both_forms(lambda dt: ops.kbt_gemm_mul_leakyrelu(dev(x, dt), dev(w, dt), dev(b, torch.float32), 1.5, 0.01,
                                                     out_dtype=dt), ref, what="mul_leakyrelu")


@pytest.mark.parametrize("M,N,K", SHAPES + [(40, 4096, 128)])
def test_kbt_gemm_div_sum_scale(oracle, M, N, K):
    rng = np.random.default_rng(5 * M + K)
    x, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    ref = oracle.kbt_gemm_div_sum_scale(x, w, M, N, K, 2.0)
    both_forms(lambda dt: ops.kbt_gemm_div_sum_scale(dev(x, dt), dev(w, dt), 2.0, out_dtype=torch.float32), ref,
               rows=False, what="div_sum_scale")


@pytest.mark.parametrize("M,N,K", ROW_SHAPES + [(200, 264, 136)])
def test_kbt_gemm_layernorm(oracle, M, N, K):
    rng = np.random.default_rng(11 * M + N)
    x, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    b = rng.standard_normal(N).astype(np.float32) * 0.02
    g = (1 + rng.standard_normal(N) * 0.02).astype(np.float32)
    beta = rng.standard_normal(N).astype(np.float32) * 0.02
    ref = oracle.kbt_gemm_layernorm(x, w, b, g, beta, M, N, K, 1e-5)
    f32 = torch.float32
    both_forms(lambda dt: ops.kbt_gemm_layernorm(dev(x, dt), dev(w, dt), dev(b, f32), dev(g, f32), dev(beta, f32),
                                                 1e-5, out_dtype=dt), ref, what="layernorm")


# D <= 256 runs the fused two-sweep kernel (softmax_rows_kernel); larger D the
# GEMM with stored scores plus the finaliser.
@pytest.mark.parametrize("M,N,D", [(16, 16, 8), (24, 40, 16), (200, 264, 64), (72, 1048, 128), (40, 4096, 128),
                                   (520, 1000, 128), (136, 264, 256), (72, 520, 264)])
def test_kbt_attention_score(oracle, M, N, D):
    rng = np.random.default_rng(13 * M + N)
    q, k = f16(rng, (M, D)), f16(rng, (N, D))
    ref = oracle.kbt_attention_score(q, k, M, N, D)
    both_forms(lambda dt: ops.kbt_attention_score(dev(q, dt), dev(k, dt), out_dtype=dt), ref, what="attn_score")


# K <= 256 is fused (both sweeps recompute the product); (136, 520, 1032) and
# (264, 1040, 320) take the stored-scores path; 19456 rows are 152 row blocks,
# more than one per SM.
@pytest.mark.parametrize("M,N,K", ROW_SHAPES + [(200, 264, 136), (136, 520, 1032), (264, 1040, 320),
                                                (19456, 264, 64)])
def test_kbt_matmul_softmax(oracle, M, N, K):
    rng = np.random.default_rng(17 * M + N)
    a, b = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    ref = oracle.kbt_matmul_softmax(a, b, M, N, K)
    both_forms(lambda dt: ops.kbt_matmul_softmax(dev(a, dt), dev(b, dt), out_dtype=dt), ref, what="softmax")


@pytest.mark.parametrize("M,N,K", ROW_SHAPES + [(200, 264, 136)])
@pytest.mark.parametrize("with_temp", [False, True])
def test_kbt_matmul_scale_residadd_clamp(oracle, M, N, K, with_temp):
    rng = np.random.default_rng(19 * M + N)
    a, b = f16(rng, (M, K)), f16(rng, (K, N), 2 * K ** -0.5)  # wide enough that the clamp is active
    ref = oracle.kbt_matmul_scale_residadd_clamp(a, b, M, N, K, 0.5, -2.0, 2.0)

    def run(dt):
        temp = torch.empty((M, N), device="cuda", dtype=torch.float32) if with_temp else None
        return ops.kbt_matmul_scale_residadd_clamp(dev(a, dt), dev(b, dt), 0.5, -2.0, 2.0, temp=temp)
    both_forms(run, ref, rows=False, what="clamp_lse_mish")


@pytest.mark.parametrize("M,N,K", SHAPES + [(40, 4096, 128)])
def test_kbt_matmul_sum_max_avgpool(oracle, M, N, K):
    rng = np.random.default_rng(23 * M + N)
    x, w, b = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5), rng.standard_normal(N).astype(np.float32) * 0.1
    ref = oracle.kbt_matmul_sum_max_avgpool(x, w, b, M, N, K)
    both_forms(lambda dt: ops.kbt_matmul_sum_max_avgpool(dev(x, dt), dev(w, dt), dev(b, torch.float32)), ref,
               rows=False, what="sum")


@pytest.mark.parametrize("M,N,K", SHAPES)
@pytest.mark.parametrize("with_norm", [False, True])
def test_kbt_gemm_rmsnorm_swiglu(oracle, M, N, K, with_norm):
    rng = np.random.default_rng(29 * M + N)
    x = f16(rng, (M, K))
    rw = (1 + rng.standard_normal(K) * 0.02).astype(np.float32)
    wg, wu = f16(rng, (K, N), K ** -0.5), f16(rng, (K, N), K ** -0.5)
    ref = oracle.kbt_gemm_rmsnorm_swiglu(x, rw, wg, wu, M, N, K, 1e-6)

    def run(dt):
        norm = torch.empty((M, K), device="cuda", dtype=torch.float32) if with_norm else None
        return ops.kbt_gemm_rmsnorm_swiglu(dev(x, dt), dev(rw, torch.float32), dev(wg, dt), dev(wu, dt), 1e-6,
                                           norm=norm, out_dtype=dt)
    both_forms(run, ref, what="rmsnorm_swiglu")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kbt_gemm_silu_mul(oracle, M, N, K):
    rng = np.random.default_rng(31 * M + N)
    x = f16(rng, (M, K))
    wa, wb = f16(rng, (K, N), K ** -0.5), f16(rng, (K, N), K ** -0.5)
    ba, bb = (rng.standard_normal(N) * 0.02).astype(np.float32), (rng.standard_normal(N) * 0.02).astype(np.float32)
    ref = oracle.kbt_gemm_silu_mul(x, wa, ba, wb, bb, M, N, K)
    f32 = torch.float32
    both_forms(lambda dt: ops.kbt_gemm_silu_mul(dev(x, dt), dev(wa, dt), dev(ba, f32), dev(wb, dt), dev(bb, f32),
                                                out_dtype=dt), ref, what="silu_mul")


def test_known_answers_identity_ones_zero():
    """GEMM known answers (the cupbop_gemm checks: A.I = A, ones.ones = K, A.0 = 0)."""
    M = N = K = 64
    rng = np.random.default_rng(0)
    a = f16(rng, (M, K))
    eye = np.eye(K, N, dtype=np.float32)
    got = ops.kbt_sgemm(dev(a, torch.float16), dev(eye, torch.float16)).cpu().numpy()
    assert np.array_equal(got, a)
    ones = np.ones((M, K), np.float32)
    got = ops.kbt_sgemm(dev(ones, torch.float16), dev(ones, torch.float16)).cpu().numpy()
    assert (got == K).all()
    got = ops.kbt_sgemm(dev(a, torch.float16), dev(np.zeros((K, N), np.float32), torch.float16)).cpu().numpy()
    assert not got.any()


def test_softmax_constant_and_one_hot_rows():
    """Softmax known answers (cupbop_softmax checks): constant row -> uniform, dominant entry -> one-hot."""
    M, N, K = 16, 512, 16
    a = np.zeros((M, K), np.float32)
    a[:, 0] = 1.0
    b = np.zeros((K, N), np.float32)
    got = ops.kbt_matmul_softmax(dev(a, torch.float16), dev(b, torch.float16), out_dtype=torch.float32).cpu().numpy()
    np.testing.assert_allclose(got, 1.0 / N, rtol=1e-5)
    b[0, 7] = 60.0
    got = ops.kbt_matmul_softmax(dev(a, torch.float16), dev(b, torch.float16), out_dtype=torch.float32).cpu().numpy()
    np.testing.assert_allclose(got[:, 7], 1.0, rtol=1e-5)


def test_m_zero_is_a_noop_and_launch_counter_moves():
    before = ops.launch_count()
    x = torch.zeros((0, 64), device="cuda", dtype=torch.float16)
    w = torch.zeros((64, 64), device="cuda", dtype=torch.float16)
    b = torch.zeros(64, device="cuda", dtype=torch.float32)
    out = ops.kbt_gemm_add_relu(x, w, b)
    assert out.shape == (0, 64)
    assert ops.launch_count() == before
    ops.kbt_gemm_add_relu(torch.zeros((8, 64), device="cuda", dtype=torch.float16), w, b)
    assert ops.launch_count() > before


def test_workspace_too_small_is_rejected_and_exact_fit_works(oracle):
    from akili_bench_b200 import abi
    M, N, K = 64, 4096, 64
    rng = np.random.default_rng(4)
    x, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    b, g, beta = (np.zeros(N, np.float32), np.ones(N, np.float32), np.zeros(N, np.float32))
    arg = abi.KbtGemmLayernormArg()
    arg.M, arg.N, arg.K, arg.eps = M, N, K, 1e-5
    ex = abi.make_ex(abi.DTYPE_F16, abi.DTYPE_F16)
    import ctypes as C
    need = C.c_uint64(0)
    assert abi.load().akili_workspace_bytes(b"kbt_gemm_layernorm", C.byref(arg), C.byref(ex), C.byref(need)) == 0
    assert need.value > 0
    f32 = torch.float32
    small = torch.empty(int(need.value) // 4 - 64, device="cuda", dtype=f32)
    with pytest.raises(abi.AkiliError) as e:
        ops.kbt_gemm_layernorm(dev(x, torch.float16), dev(w, torch.float16), dev(b, f32), dev(g, f32), dev(beta, f32),
                               workspace=small)
    assert e.value.code == abi.E_WORKSPACE
    ws = torch.empty(int(need.value) // 4, device="cuda", dtype=f32)
    got = ops.kbt_gemm_layernorm(dev(x, torch.float16), dev(w, torch.float16), dev(b, f32), dev(g, f32),
                                 dev(beta, f32), workspace=ws).float().cpu().numpy()
    assert_parity(got, oracle.kbt_gemm_layernorm(x, w, b, g, beta, M, N, K, 1e-5))


# Row-fused LayerNorm / softmax (CTA-pair kernel, M > 128): the epilogue merges
# each row's statistics across the CTAs of the row block and stores the
# normalised row once, one launch.  AKILI_ROWNORM=0 selects the two-pass form
# (GEMM with statistics, then a finaliser: two launches).  Shapes: ragged M and
# N, several row blocks whose tiles straddle a wave, N of 33 tiles, and N of 75
# tiles (more than one wave of CTA pairs holds: the two-pass form either way).
ROWFUSED = [(264, 4104, 136), (200, 264, 136), (520, 8200, 264), (2056, 4096, 256), (1032, 1048, 520),
            (264, 18952, 64)]


@pytest.mark.parametrize("M,N,K", ROWFUSED)
@pytest.mark.parametrize("mode", ["1", "0"])
def test_layernorm_row_fused_and_two_pass(oracle, monkeypatch, M, N, K, mode):
    monkeypatch.setenv("AKILI_ROWNORM", mode)
    rng = np.random.default_rng(23 * M + N)
    x, w = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5)
    b = rng.standard_normal(N).astype(np.float32) * 0.02
    g = (1 + rng.standard_normal(N) * 0.02).astype(np.float32)
    beta = rng.standard_normal(N).astype(np.float32) * 0.02
    ref = oracle.kbt_gemm_layernorm(x, w, b, g, beta, M, N, K, 1e-5, threads=8)
    f16t, f32 = torch.float16, torch.float32
    args = (dev(x, f16t), dev(w, f16t), dev(b, f32), dev(g, f32), dev(beta, f32))
    for odt in (f16t, f32):
        torch.cuda.synchronize()
        l0 = ops.launch_count()
        got = ops.kbt_gemm_layernorm(*args, 1e-5, out_dtype=odt).float().cpu().numpy()
        launches = ops.launch_count() - l0
        assert ops.device_status() == 0
        assert_parity(got, ref, what=f"layernorm rownorm={mode} {odt}")
        assert launches == (1 if mode != "0" and N <= 74 * 256 else 2)


@pytest.mark.parametrize("M,N,K", [(264, 1040, 320), (1032, 4096, 512), (2056, 2056, 264), (520, 8200, 264)])
@pytest.mark.parametrize("mode", ["1", "0"])
def test_matmul_softmax_row_fused_and_two_pass(oracle, monkeypatch, M, N, K, mode):
    monkeypatch.setenv("AKILI_ROWNORM", mode)
    rng = np.random.default_rng(29 * M + N)
    a, b = f16(rng, (M, K)), f16(rng, (K, N), K ** -0.5 * 3)
    ref = oracle.kbt_matmul_softmax(a, b, M, N, K, threads=8)
    f16t = torch.float16
    for odt in (f16t, torch.float32):
        torch.cuda.synchronize()
        l0 = ops.launch_count()
        got = ops.kbt_matmul_softmax(dev(a, f16t), dev(b, f16t), out_dtype=odt).float().cpu().numpy()
        launches = ops.launch_count() - l0
        assert ops.device_status() == 0
        assert_parity(got, ref, what=f"softmax rownorm={mode} {odt}")
        np.testing.assert_allclose(got.sum(1), 1.0, rtol=2e-3)
        assert launches == (1 if mode != "0" else 2)
