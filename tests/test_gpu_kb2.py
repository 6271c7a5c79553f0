"""GPU parity of the kb2_* family (fp32 operands, fp32 arithmetic) against the
CPU oracle's restatement of each kb2 gold loop.

The kb2 entries keep fp32 semantics: no fp16 rounding of the operands (the
GEMM runs on the tensor cores over fp16 hi + lo parts of each operand).  So
beside the parity bar of the kbt tests (max|err| <= 1e-2 * max|ref|, row
cosine >= 0.9999) every case must also agree to fp32 level:
max|err| <= 1e-4 * max|ref|.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import abi  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402
from golden_cases import case_files, load_case, oracle_eval  # noqa: E402

pytestmark = pytest.mark.gpu

SHAPES = [(16, 16, 16), (24, 40, 56), (200, 264, 136), (136, 520, 1032)]


def dev(x):
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).cuda()


def call(op, out_shape, bufs, **scalars):
    """akili_<op> through the C ABI: fp32 device buffers named like the
    reference struct's *_addr fields, plus its scalar fields."""
    st = abi.OPS[op][0]()
    for k, v in scalars.items():
        setattr(st, k, v)
    keep = {k: dev(v) for k, v in bufs.items()}
    for k, t in keep.items():
        setattr(st, f"{k}_addr", t.data_ptr())
    out = torch.zeros(out_shape, device="cuda", dtype=torch.float32)
    st.c_addr = out.data_ptr()
    abi.check(op, st)
    torch.cuda.synchronize()
    v = C.c_uint32(0)
    assert abi.load().akili_device_status(C.byref(v), 1) == abi.OK
    return out.cpu().numpy()


def check(got, ref, rows=True, what=""):
    assert_parity(got, ref, rows=rows, what=what)
    scale = float(np.abs(ref).max()) or 1.0
    err = float(np.abs(got - ref).max())
    assert err <= 1e-4 * scale, f"{what}: max|err| {err:.3e} > 1e-4 * {scale:.3e} (fp32-level accuracy)"


def rnd(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float32)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_add_relu(oracle, M, N, K):
    rng = np.random.default_rng(M + N + K)
    a, w, b = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5), rnd(rng, N, 0.1)
    got = call("kb2_gemm_add_relu", (M, N), {"a": a, "w": w, "bias": b}, M=M, N=N, K=K)
    check(got, oracle.kb2_gemm_add_relu(a, w, b, M, N, K), what="kb2 add_relu")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_mul_leakyrelu(oracle, M, N, K):
    rng = np.random.default_rng(2 * M + N)
    a, w, b = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5), rnd(rng, N, 0.1)
    got = call("kb2_gemm_mul_leakyrelu", (M, N), {"a": a, "w": w, "bias": b}, M=M, N=N, K=K, multiplier=1.5,
               negative_slope=0.01)
    check(got, oracle.kb2_gemm_mul_leakyrelu(a, w, b, M, N, K, 1.5, 0.01), what="kb2 mul_leakyrelu")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_div_sum_scale(oracle, M, N, K):
    rng = np.random.default_rng(3 * M + N)
    a, w = rnd(rng, (M, K), 1.0), rnd(rng, (K, N), K ** -0.5) + 0.05
    got = call("kb2_gemm_div_sum_scale", (M,), {"a": a, "w": w}, M=M, N=N, K=K, scaling_factor=2.0)
    check(got, oracle.kb2_gemm_div_sum_scale(a, w, M, N, K, 2.0), rows=False, what="kb2 div_sum_scale")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_layernorm(oracle, M, N, K):
    rng = np.random.default_rng(4 * M + N)
    a, w, b = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5), rnd(rng, N, 0.1)
    g, beta = 1.0 + rnd(rng, N, 0.02), rnd(rng, N, 0.02)
    got = call("kb2_gemm_layernorm", (M, N), {"a": a, "w": w, "bias": b, "ln_w": g, "ln_b": beta}, M=M, N=N, K=K,
               eps=1e-5)
    check(got, oracle.kb2_gemm_layernorm(a, w, b, g, beta, M, N, K, 1e-5), what="kb2 layernorm")


@pytest.mark.parametrize("M,N,D", [(16, 16, 16), (24, 40, 16), (200, 264, 64), (72, 1048, 128)])
def test_kb2_attention_score(oracle, M, N, D):
    rng = np.random.default_rng(5 * M + N)
    q, k = rnd(rng, (M, D)), rnd(rng, (N, D))
    got = call("kb2_attention_score", (M, N), {"q": q, "k": k}, M=M, N=N, D=D)
    check(got, oracle.kb2_attention_score(q, k, M, N, D), what="kb2 attention_score")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_matmul_softmax(oracle, M, N, K):
    rng = np.random.default_rng(6 * M + N)
    a, w = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5)
    got = call("kb2_matmul_softmax", (M, N), {"a": a, "b": w}, M=M, N=N, K=K)
    check(got, oracle.kb2_matmul_softmax(a, w, M, N, K), what="kb2 matmul_softmax")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_matmul_scale_residadd_clamp(oracle, M, N, K):
    rng = np.random.default_rng(7 * M + N)
    a, w, b = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5), rnd(rng, N, 0.1)
    got = call("kb2_matmul_scale_residadd_clamp", (M,), {"a": a, "w": w, "bias": b}, M=M, N=N, K=K,
               scale_factor=2.0, clamp_min=-10.0, clamp_max=10.0)
    check(got, oracle.kb2_matmul_scale_residadd_clamp(a, w, b, M, N, K, 2.0, -10.0, 10.0), rows=False,
          what="kb2 clamp")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_matmul_sum_max_avgpool(oracle, M, N, K):
    rng = np.random.default_rng(8 * M + N)
    a, w, b = rnd(rng, (M, K)), rnd(rng, (K, N), K ** -0.5) + 0.05, rnd(rng, N, 0.1)
    got = call("kb2_matmul_sum_max_avgpool", (M,), {"a": a, "w": w, "bias": b}, M=M, N=N, K=K)
    check(got, oracle.kb2_matmul_sum_max_avgpool(a, w, b, M, N, K), rows=False, what="kb2 sum_max_avgpool")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_rmsnorm_swiglu(oracle, M, N, K):
    rng = np.random.default_rng(9 * M + N)
    x, rw = rnd(rng, (M, K)), 1.0 + rnd(rng, K, 0.02)
    wg, wu = rnd(rng, (K, N), K ** -0.5), rnd(rng, (K, N), K ** -0.5)
    got = call("kb2_gemm_rmsnorm_swiglu", (M, N), {"x": x, "rms_w": rw, "wg": wg, "wu": wu}, M=M, N=N, K=K,
               eps=1e-5)
    check(got, oracle.kb2_gemm_rmsnorm_swiglu(x, rw, wg, wu, M, N, K, 1e-5), what="kb2 rmsnorm_swiglu")


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_kb2_gemm_silu_mul(oracle, M, N, K):
    rng = np.random.default_rng(10 * M + N)
    a = rnd(rng, (M, K))
    wa, wb = rnd(rng, (K, N), K ** -0.5), rnd(rng, (K, N), K ** -0.5)
    ba, bb = rnd(rng, N, 0.02), rnd(rng, N, 0.02)
    got = call("kb2_gemm_silu_mul", (M, N), {"a": a, "wa": wa, "ba": ba, "wb": wb, "bb": bb}, M=M, N=N, K=K)
    check(got, oracle.kb2_gemm_silu_mul(a, wa, ba, wb, bb, M, N, K), what="kb2 silu_mul")


@pytest.mark.parametrize("path", [p for p in case_files() if p.split("/")[-1].startswith("kb2_")],
                         ids=lambda p: p.split("/")[-1][:-4])
def test_kb2_golden_vectors(oracle, path):
    """The reference harness's own inputs through akili_kb2_*, against its gold."""
    bench, arg, d = load_case(path)
    bufs = {k: torch.from_numpy(v).cuda() for k, v in d.items() if k not in ("expected", "argv")}
    out = torch.zeros(d["expected"].size, device="cuda")
    for name, t in bufs.items():
        setattr(arg, f"{name}_addr", t.data_ptr())
    arg.c_addr = out.data_ptr()
    abi.check(bench, arg)
    torch.cuda.synchronize()
    got = out.cpu().numpy()
    ref = d["expected"]
    assert np.array_equal(oracle_eval(oracle, bench, arg, d), ref)  # the oracle is the gold, bit for bit
    rows = ref.size != arg.M
    check(got.reshape((arg.M, -1) if rows else (-1,)), ref.reshape((arg.M, -1) if rows else (-1,)), rows=rows,
          what=bench)
