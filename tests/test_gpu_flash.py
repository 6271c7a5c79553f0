"""GPU parity of the flash-attention forward against the CPU oracle.

The plain entry (akili_flash) is the reference's semantics: one head,
Q/K/V/O fp32 [seq_len x head_dim], no softmax scale.  The _ex entry adds
batch x heads ([B, H, S, D] fp16) and the 1/sqrt(d) scale of the benchmark
configuration.  Operands are fp16-rounded once so both sides see the same
values.  Tolerance: max|err| <= 1e-2 * max|ref| and per-row cosine >= 0.9999.
"""
import ctypes as C
import os

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu


def f16(rng, shape, scale=1.0):
    return (rng.standard_normal(shape, dtype=np.float32) * scale).astype(np.float16).astype(np.float32)


def dev(x, dtype):
    return torch.from_numpy(np.ascontiguousarray(x)).to("cuda", dtype)


@pytest.mark.parametrize("S,D", [(16, 8), (64, 8), (128, 16), (200, 64), (256, 128), (384, 96), (1000, 32)])
def test_flash_reference_semantics_one_head(oracle, S, D):
    """akili_flash: fp32 in/out, unscaled softmax, one head (benchmarks/flash/main.cpp:52-85)."""
    rng = np.random.default_rng(S + D)
    q, k, v = f16(rng, (S, D), 0.5), f16(rng, (S, D), 0.5), f16(rng, (S, D))
    ref = oracle.flash(q, k, v, S, D, 1.0)
    got = ops.flash(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32)).cpu().numpy()
    assert ops.device_status() == 0
    assert_parity(got, ref, what=f"flash S={S} D={D}")


@pytest.mark.parametrize("B,H,S,D", [(1, 2, 128, 128), (2, 3, 320, 64), (1, 2, 1024, 128), (2, 1, 136, 8)])
@pytest.mark.parametrize("out_dtype", ["f16", "f32"])
def test_flash_batched_scaled_fp16(oracle, B, H, S, D, out_dtype):
    rng = np.random.default_rng(B * 1000 + S)
    q, k, v = f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D))
    scale = D ** -0.5
    odt = torch.float16 if out_dtype == "f16" else torch.float32
    got = ops.flash(dev(q, torch.float16), dev(k, torch.float16), dev(v, torch.float16), softmax_scale=scale,
                    out_dtype=odt).float().cpu().numpy()
    assert ops.device_status() == 0
    for b in range(B):
        for h in range(H):
            ref = oracle.flash(q[b, h].copy(), k[b, h].copy(), v[b, h].copy(), S, D, scale)
            assert_parity(got[b, h], ref, what=f"flash b={b} h={h}")


def test_flash_known_answers():
    """cupbop_fmha checks: identical query rows give identical output rows;
    V = I (S == D) returns the softmax weights themselves."""
    S = D = 128
    rng = np.random.default_rng(7)
    q = np.repeat(f16(rng, (1, D)), S, axis=0)
    k = f16(rng, (S, D))
    v = np.eye(S, D, dtype=np.float32)
    got = ops.flash(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32)).cpu().numpy()
    assert np.allclose(got, got[0:1], atol=0)
    np.testing.assert_allclose(got.sum(1), 1.0, rtol=2e-3)


def test_flash_large_logits_are_stable(oracle):
    """Scores in the hundreds (reference harness inputs: uniform [-5, 5), d=8, no scale)."""
    S, D = 256, 8
    rng = np.random.default_rng(3)
    q = (rng.random((S, D), dtype=np.float32) * 10 - 5).astype(np.float16).astype(np.float32)
    k = (rng.random((S, D), dtype=np.float32) * 10 - 5).astype(np.float16).astype(np.float32)
    v = (rng.random((S, D), dtype=np.float32) * 10 - 5).astype(np.float16).astype(np.float32)
    ref = oracle.flash(q, k, v, S, D, 1.0)
    got = ops.flash(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32)).cpu().numpy()
    assert_parity(got, ref, what="flash large logits")


@pytest.mark.parametrize("S,D", [(256, 8), (128, 16), (300, 64)])
def test_flash_fp32_simt_mode_matches_unrounded_gold(oracle, S, D):
    """kernel_type 0 with fp32 inputs (the reference SIMT flash, fp32
    arithmetic): split-precision scores track the fp32 gold on the reference
    harness's own input range (uniform [-5, 5), no scale: logits in the
    hundreds), where fp16-rounded scores would not."""
    rng = np.random.default_rng(S * 3 + D)
    q, k, v = (rng.random((S, D), dtype=np.float32) * 10 - 5 for _ in range(3))
    ref = oracle.flash(q, k, v, S, D, 1.0)
    got = ops.flash(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32), kernel_type=0).cpu().numpy()
    assert ops.device_status() == 0
    assert_parity(got, ref, what=f"flash fp32 simt S={S} D={D}")
    # and the reference harness's own per-element bound (flash/main.cpp:37-49)
    assert (np.abs(got - ref) <= 5e-2 + 1e-2 * np.abs(got)).all()


def _heads(oracle, q, k, v, scale, causal):
    B, H, S, D = q.shape
    o = np.zeros_like(q)
    m = np.zeros((B, H, S), np.float32)
    l = np.zeros((B, H, S), np.float32)
    for b in range(B):
        for h in range(H):
            o[b, h], m[b, h], l[b, h] = oracle.flash_causal(q[b, h].copy(), k[b, h].copy(), v[b, h].copy(), S, D,
                                                            scale, causal=causal)
    return o, m, l


# S values that are not multiples of the 256-query CTA tile or the 128-key
# block exercise the diagonal and the tails together.
@pytest.mark.parametrize("B,H,S,D", [(1, 2, 256, 128), (2, 1, 300, 64), (1, 1, 520, 128), (1, 3, 136, 8),
                                     (1, 1, 1024, 128)])
@pytest.mark.parametrize("causal", [True, False])
def test_flash_causal_and_row_statistics(oracle, B, H, S, D, causal):
    """cupbop_dao_flash semantics (key j > query i masked) and the m/l row
    statistics of its kernel, against the oracle on the same fp16 operands."""
    rng = np.random.default_rng(B * 100 + S + D + causal)
    q, k, v = f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D))
    scale = D ** -0.5
    ref_o, ref_m, ref_l = _heads(oracle, q, k, v, scale, causal)
    got_o, got_m, got_l = ops.flash(dev(q, torch.float16), dev(k, torch.float16), dev(v, torch.float16),
                                    softmax_scale=scale, out_dtype=torch.float32, causal=causal, return_stats=True)
    assert ops.device_status() == 0
    got_o = got_o.cpu().numpy()
    for b in range(B):
        for h in range(H):
            assert_parity(got_o[b, h], ref_o[b, h], what=f"flash causal={causal} b={b} h={h}")
    np.testing.assert_allclose(got_m.cpu().numpy(), ref_m, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got_l.cpu().numpy(), ref_l, rtol=2e-3)
    if causal:  # the first query sees only the first key
        np.testing.assert_allclose(got_o[:, :, 0], v[:, :, 0], rtol=0, atol=1e-6)
        np.testing.assert_allclose(got_l.cpu().numpy()[:, :, 0], 1.0, rtol=1e-6)


def test_flash_causal_fp32_reference_semantics(oracle):
    """fp32 buffers with the fp32 SIMT kernel type (split-precision scores),
    unscaled, one head, causal: held to the unrounded fp32 oracle."""
    S, D = 200, 16
    rng = np.random.default_rng(11)
    q, k, v = (rng.standard_normal((S, D), dtype=np.float32) for _ in range(3))
    ref_o, ref_m, ref_l = oracle.flash_causal(q, k, v, S, D, 1.0, causal=True)
    got_o, got_m, got_l = ops.flash(dev(q, torch.float32), dev(k, torch.float32), dev(v, torch.float32),
                                    kernel_type=0, causal=True, return_stats=True)
    assert ops.device_status() == 0
    assert_parity(got_o.cpu().numpy(), ref_o, what="flash causal fp32")
    np.testing.assert_allclose(got_m.cpu().numpy(), ref_m, rtol=1e-4, atol=1e-4)
    np.testing.assert_allclose(got_l.cpu().numpy(), ref_l, rtol=2e-3)


# ---- the m / l statistics against the reference's own causal flash kernel ----

DAO_LIB = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "oracle", "_ref",
                       "libdao_flash_ref.so")


def _dao_lib():
    if not os.path.exists(DAO_LIB):
        pytest.skip("reference-built libdao_flash_ref.so not present (python oracle/build_oracle.py)")
    return C.CDLL(DAO_LIB)


def test_reference_dao_flash_kernel_passes_its_own_tests():
    """The reference's CUDA kernel dao_flash_fwd, built unchanged from
    cupbop_dao_flash/dao_flash_cupbop.cu, passes the reference's own eight
    tests (its main(), :246-345) on this GPU before it serves as a pin."""
    assert _dao_lib().akili_ref_dao_selftest() == 0


# Bc = Br threads per block and N a multiple of Bc: the reference kernel's
# own launch conditions (dao_flash_cupbop.cu:216-222), checked by the wrapper.
@pytest.mark.parametrize("B,H,S,D,Bc", [(1, 1, 8, 8, 8), (1, 2, 64, 64, 16), (2, 2, 256, 128, 16),
                                        (1, 1, 512, 64, 32), (1, 3, 136, 8, 8)])
@pytest.mark.parametrize("causal", [0, 1])
def test_flash_stats_match_reference_kernel(oracle, B, H, S, D, Bc, causal):
    """akili_flash_ml_ex's O, m and l against the m / l / O buffers of the
    reference kernel dao_flash_fwd (online softmax over Bc-key tiles,
    dao_flash_cupbop.cu:79-131: m = running max of the scaled scores, l =
    sum exp(score - m) rescaled tile by tile), both on the same fp16-rounded
    operands with the reference's scale 1/sqrt(d).  The oracle's m is the
    same maximum, so it is checked against the reference kernel too."""
    lib = _dao_lib()
    rng = np.random.default_rng(S * 5 + D + causal)
    q, k, v = f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D)), f16(rng, (B, H, S, D))
    scale = float(np.float32(1.0) / np.sqrt(np.float32(D)))
    ro, rm, rl = np.zeros_like(q), np.zeros((B, H, S), np.float32), np.zeros((B, H, S), np.float32)
    f = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    rc = lib.akili_ref_dao_flash_fwd(f(q), f(k), f(v), f(ro), f(rm), f(rl), B, H, S, D, Bc, C.c_float(scale),
                                     causal)
    assert rc == 0
    got_o, got_m, got_l = ops.flash(dev(q, torch.float16), dev(k, torch.float16), dev(v, torch.float16),
                                    softmax_scale=scale, out_dtype=torch.float32, causal=bool(causal),
                                    return_stats=True)
    assert ops.device_status() == 0
    got_o = got_o.cpu().numpy()
    for b in range(B):
        for h in range(H):
            assert_parity(got_o[b, h], ro[b, h], what=f"flash vs dao_flash_fwd b={b} h={h}")
    np.testing.assert_allclose(got_m.cpu().numpy(), rm, rtol=1e-5, atol=1e-5)
    np.testing.assert_allclose(got_l.cpu().numpy(), rl, rtol=2e-3)
    _, om, ol = _heads(oracle, q, k, v, scale, bool(causal))
    np.testing.assert_allclose(om, rm, rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(ol, rl, rtol=1e-5)
