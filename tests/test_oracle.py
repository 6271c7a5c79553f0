"""The CPU oracle against akili-bench's own gold (CPU only).

Two independent pins:
1. the golden vectors of tests/golden/ (captured from the reference harness's
   own verify loop) must equal the oracle bit for bit;
2. where the reference-built pin binaries exist (oracle/_ref/pin/, built by
   oracle/build_oracle.py from the unchanged reference main.cpp), the
   reference harness itself, with its verify loop turned into an exact
   comparison, must print PASSED! at several sizes — and FAILED! when the
   stand-in device returns zeros or a 1-ulp-perturbed oracle output.
"""
import os
import subprocess

import numpy as np
import pytest

from golden_cases import case_files, load_case, oracle_eval

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PIN = os.path.join(ROOT, "oracle", "_ref", "pin")

BENCHES = ["kbt_sgemm", "kbt_gemm_add_relu", "kbt_gemm_mul_leakyrelu", "kbt_gemm_div_sum_scale",
           "kbt_gemm_layernorm", "kbt_attention_score", "kbt_matmul_softmax",
           "kbt_matmul_scale_residadd_clamp", "kbt_matmul_sum_max_avgpool", "kbt_gemm_rmsnorm_swiglu",
           "kbt_gemm_silu_mul", "flash"]
KB2 = ["kb2_gemm_add_relu", "kb2_gemm_mul_leakyrelu", "kb2_gemm_div_sum_scale", "kb2_gemm_layernorm",
       "kb2_attention_score", "kb2_matmul_softmax", "kb2_matmul_scale_residadd_clamp",
       "kb2_matmul_sum_max_avgpool", "kb2_gemm_rmsnorm_swiglu", "kb2_gemm_silu_mul"]


def test_every_bench_has_golden_cases():
    for b in BENCHES + KB2:
        assert len(case_files(b)) >= 3, b


@pytest.mark.parametrize("path", case_files(), ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_bit_exact_vs_reference_golden(oracle, path):
    bench, arg, d = load_case(path)
    got = oracle_eval(oracle, bench, arg, d)
    exp = d["expected"]
    assert got.shape == exp.shape
    # bit-exact: compare the raw fp32 patterns (+0/-0 are the only tolerated difference)
    same = (got.view(np.uint32) == exp.view(np.uint32)) | ((got == 0) & (exp == 0))
    assert same.all(), f"{(~same).sum()} of {same.size} differ; first at {np.argmax(~same)}"


def test_row_subset_and_threads_match_full(oracle):
    rng = np.random.default_rng(1)
    M, N, K = 40, 24, 72
    a = rng.standard_normal((M, K), dtype=np.float32)
    w = rng.standard_normal((K, N), dtype=np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    full = oracle.kbt_gemm_add_relu(a, w, b, M, N, K)
    part = oracle.kbt_gemm_add_relu(a, w, b, M, N, K, row0=8, row1=33, threads=4)
    assert np.array_equal(full[8:33], part[8:33])
    assert not part[:8].any() and not part[33:].any()


def test_round_f16_matches_numpy(oracle):
    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal(10000).astype(np.float32) * s for s in (1e-6, 1e-3, 1, 1e3, 6e4)])
    x = np.concatenate([x, np.float32([65504, 65519.99, 65520, -70000, 2**-24, 2**-25, 3 * 2**-26, 0.0, -0.0])])
    assert np.array_equal(oracle.round_f16(x), x.astype(np.float16).astype(np.float32))


PIN_SIZES = {
    "default": [],
    "odd": ["-m24", "-n40", "-p56"],
    "tall": ["-m72", "-n16", "-p8"],
    "unaligned_flags": ["-m13", "-n9", "-p21"],  # rounded up to multiples of 8 by the harness
}
PIN_FLASH = [["-n", "64", "-d", "8", "-t", "1"], ["-n", "256", "-d", "8", "-t", "1"],
             ["-n", "128", "-d", "16", "-t", "0"], ["-n", "32", "-d", "4", "-t", "0"]]


def _pin(bench, argv, **env):
    exe = os.path.join(PIN, bench)
    if not os.path.exists(exe):
        pytest.skip("reference-built pin binaries not present (python oracle/build_oracle.py)")
    e = dict(os.environ, AKILI_PROBE="exact", **env)
    r = subprocess.run([exe, *argv], env=e, capture_output=True, text=True, timeout=120)
    return r.returncode, r.stdout


@pytest.mark.parametrize("bench", [b for b in BENCHES if b != "flash"] + KB2)
@pytest.mark.parametrize("size", list(PIN_SIZES))
def test_reference_harness_exact_pin(bench, size):
    argv = PIN_SIZES[size]
    if bench in ("kbt_attention_score", "kb2_attention_score"):
        argv = [a.replace("-p", "-d") for a in argv]
    rc, out = _pin(bench, argv)
    assert rc == 0 and "PASSED!" in out, out[-400:]


@pytest.mark.parametrize("argv", PIN_FLASH, ids=lambda a: "".join(a).replace("-", "_"))
def test_reference_flash_harness_exact_pin(argv):
    rc, out = _pin("flash", argv)
    assert rc == 0 and "PASSED!" in out, out[-400:]


@pytest.mark.parametrize("bench", ["kbt_gemm_add_relu", "kbt_gemm_layernorm", "flash", "kb2_gemm_add_relu",
                                   "kb2_matmul_softmax"])
def test_exact_pin_negative_controls(bench):
    argv = ["-n", "64", "-d", "8", "-t", "1"] if bench == "flash" else []
    # (the harness returns its error count, which can wrap to exit status 0: read the text)
    rc, out = _pin(bench, argv, AKILI_HOST_DEVICE="zero")
    assert "FAILED!" in out and "PASSED!" not in out
    rc, out = _pin(bench, argv, AKILI_HOST_DEVICE="oracle_ulp")
    assert "Found 1 errors!" in out and "FAILED!" in out


@pytest.mark.parametrize("S,D", [(1, 8), (37, 16), (130, 64)])
def test_causal_flash_oracle_known_answers(oracle, S, D):
    """dao_flash causal semantics: row 0 attends to key 0 only (O = V[0]); the
    last row sees every key (equals the non-causal row); without the mask the
    function is the plain flash oracle.  m/l are the row max and sum of exp."""
    rng = np.random.default_rng(S * 7 + D)
    q, k, v = (rng.standard_normal((S, D), dtype=np.float32) for _ in range(3))
    scale = D ** -0.5
    o_c, m_c, l_c = oracle.flash_causal(q, k, v, S, D, scale, causal=True)
    o_n, m_n, l_n = oracle.flash_causal(q, k, v, S, D, scale, causal=False)
    assert np.array_equal(o_n, oracle.flash(q, k, v, S, D, scale))
    assert np.array_equal(o_c[0], v[0])
    assert np.array_equal(o_c[-1], o_n[-1]) and m_c[-1] == m_n[-1] and l_c[-1] == l_n[-1]
    s64 = (q.astype(np.float64) @ k.astype(np.float64).T) * scale
    mask = np.triu(np.ones((S, S), bool), 1)
    s64c = np.where(mask, -np.inf, s64)
    np.testing.assert_allclose(m_c, s64c.max(1), rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(l_c, np.exp(s64c - s64c.max(1, keepdims=True)).sum(1), rtol=1e-4)
    p = np.exp(s64c - s64c.max(1, keepdims=True))
    np.testing.assert_allclose(o_c, (p / p.sum(1, keepdims=True)) @ v, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("argv", [[], ["-n", "128", "-d", "16"], ["-n", "200", "-d", "24"]],
                         ids=lambda a: "".join(a).replace("-", "_") or "default")
def test_reference_attention_harness_exact_pin(argv):
    """benchmarks/attention: all three stages exact.  Its harness resets the
    error count before the last stage, so no stage may print an error line."""
    rc, out = _pin("attention", argv)
    assert "PASSED!" in out and "*** error" not in out, out[-400:]
    rc, out = _pin("attention", argv, AKILI_HOST_DEVICE="oracle_ulp")
    assert out.count("*** error") == 3  # one moved element per stage


# ---- causal flash: the oracle against the reference's own CPU gold ----

DAO_LIB = os.path.join(ROOT, "oracle", "_ref", "libdao_flash_ref.so")
DAO_GOLDEN = sorted(f for f in os.listdir(os.path.join(ROOT, "tests", "golden")) if f.startswith("dao_flash__"))


def _dao_oracle(oracle, q, k, v, causal):
    """oracle_flash_causal head by head, with attention_cpu's own scale
    1.0f / sqrtf((float)d) (dao_flash_cupbop.cu:136) formed in fp32."""
    B, nh, N, d = q.shape
    scale = float(np.float32(1.0) / np.sqrt(np.float32(d)))
    o = np.zeros_like(q)
    for b in range(B):
        for h in range(nh):
            o[b, h] = oracle.flash_causal(q[b, h].copy(), k[b, h].copy(), v[b, h].copy(), N, d, scale,
                                          causal=causal)[0]
    return o


def _bit_equal(a, b):
    return (a.view(np.uint32) == b.view(np.uint32)) | ((a == 0) & (b == 0))


def test_dao_flash_golden_cases_cover_the_reference_tests():
    names = {f[len("dao_flash__"):-4] for f in DAO_GOLDEN}
    for n in ("noncausal_single", "noncausal_multi_tile", "noncausal_multi_head", "causal_single",
              "causal_multi_tile", "causal_multi_head"):
        assert n in names


@pytest.mark.parametrize("name", DAO_GOLDEN, ids=lambda f: f[len("dao_flash__"):-4])
def test_causal_flash_oracle_bit_exact_vs_reference_golden(oracle, name):
    """tests/golden/dao_flash__*.npz hold attention_cpu's outputs
    (cupbop_dao_flash/dao_flash_cupbop.cu:134-169), captured by
    tests/golden/make_dao_flash_golden.py; the oracle must equal them bit for bit."""
    d = np.load(os.path.join(ROOT, "tests", "golden", name))
    got = _dao_oracle(oracle, d["q"], d["k"], d["v"], int(d["causal"]))
    same = _bit_equal(got, d["expected"])
    assert same.all(), f"{(~same).sum()} of {same.size} differ"


@pytest.mark.parametrize("B,nh,N,d", [(1, 1, 1, 8), (1, 1, 33, 16), (2, 3, 64, 32), (1, 2, 57, 128), (1, 1, 64, 8)])
@pytest.mark.parametrize("causal", [0, 1])
def test_causal_flash_oracle_bit_exact_vs_reference_build(oracle, B, nh, N, d, causal):
    """The same pin live: attention_cpu compiled unchanged from the reference
    source (oracle/_ref/libdao_flash_ref.so) against the oracle, seeded
    N(0,1) operands, N up to the gold's 64-entry score array."""
    if not os.path.exists(DAO_LIB):
        pytest.skip("reference-built libdao_flash_ref.so not present (python oracle/build_oracle.py)")
    import ctypes as C
    lib = C.CDLL(DAO_LIB)
    rng = np.random.default_rng(N * 31 + d + causal)
    q, k, v = (rng.standard_normal((B, nh, N, d), dtype=np.float32) * 2 for _ in range(3))
    exp = np.zeros_like(q)
    f = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    assert lib.akili_ref_attention_cpu(f(q), f(k), f(v), f(exp), B, nh, N, d, causal) == 0
    got = _dao_oracle(oracle, q, k, v, causal)
    assert _bit_equal(got, exp).all()
    # a planted one-ulp change in the oracle's output is seen
    bad = got.copy()
    bad.view(np.uint32)[0, 0, N - 1, 0] += 1
    assert not _bit_equal(bad, exp).all()
