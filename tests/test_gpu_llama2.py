"""GPU parity of the llama2 matmul offload (benchmarks/llama2).

* akili_llama2_matmul / akili_llama2_matvec_batch against the oracle's
  restatement of llama2/matmul_kernel.cpp, fp32: the sums run in another
  order (and, for N > 1 on aligned shapes, on the tensor cores in split
  precision), so each element must agree to
  |err| <= 4e-6 * sqrt(K) * sum_k |A[i,k] * B[k,j]|, a few fp32 rounding
  errors per term at worst;
* the reference's unchanged llama.cpp on the B200: with its own vxmath.cpp
  over the Vortex shim, and with libakili_vxmath.so (resident weights,
  one launch per batched product) in its place, against its CPU matmul
  (-v 0): every position's logits within 1e-4 of the largest, the same
  greedy text.
"""
import os
import subprocess
import sys

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import abi, ops  # noqa: E402

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.path.join(ROOT, "oracle", "_ref")
TOKENS = [1, 300, 45, 67, 89, 120, 7, 333, 400, 12, 5, 77, 260, 261, 500, 3, 44, 45, 46, 47]


def bound(a, b, K):
    return 4e-6 * max(K, 1) ** 0.5 * (np.abs(a).astype(np.float64) @ np.abs(b).astype(np.float64)) + 1e-30


@pytest.mark.parametrize("M,N,K", [
    (288, 1, 288), (768, 1, 288), (288, 1, 768), (512, 1, 128), (4096, 1, 4096), (1000, 1, 11008),
    (33, 1, 7), (100, 1, 4), (3, 1, 1),            # matrix-vector, K % 4 != 0 and tiny
    (8, 1, 60000),                                 # x too large to stage in shared memory
    (300, 1, 2048), (40, 1, 4099), (12, 1, 8),     # K % 4 != 0 at length, one short row
    (5, 3, 9), (100, 20, 30), (70, 2, 4096),       # N > 1, unaligned: CUDA-core tiles
    (64, 16, 128), (24, 40, 56), (256, 64, 4096),  # N > 1, aligned: tensor cores, split precision
])
def test_llama2_matmul_matches_oracle(oracle, M, N, K):
    rng = np.random.default_rng(M * 7 + N * 3 + K)
    a = rng.standard_normal((M, K), dtype=np.float32) * np.float32(K ** -0.5)
    b = rng.standard_normal((K, N), dtype=np.float32)
    got = ops.llama2_matmul(torch.from_numpy(a).cuda(), torch.from_numpy(b if N > 1 else b[:, 0]).cuda())
    torch.cuda.synchronize()
    got = got.cpu().numpy().reshape(M, N)
    ref = oracle.llama2_matmul(a, b, M, N, K)
    err = np.abs(got.astype(np.float64) - ref)
    assert (err <= bound(a, b, K)).all(), f"max err {err.max():.3e}"


def test_llama2_matmul_unaligned_weights_and_empty_sums(oracle):
    """A weight view that starts 4 bytes past a 16-byte boundary takes the
    scalar path; K = 0 writes zeros; M = 0 does nothing."""
    rng = np.random.default_rng(5)
    M, K = 96, 64
    base = rng.standard_normal(M * K + 1, dtype=np.float32)
    x = rng.standard_normal(K, dtype=np.float32)
    w = torch.from_numpy(base).cuda()[1:].view(M, K)
    assert w.data_ptr() % 16 == 4
    got = ops.llama2_matmul(w, torch.from_numpy(x).cuda()).cpu().numpy()
    a = base[1:].reshape(M, K)
    ref = oracle.llama2_matmul(a, x.reshape(K, 1), M, 1, K)[:, 0]
    assert (np.abs(got - ref) <= bound(a, x.reshape(K, 1), K)[:, 0]).all()
    out = torch.full((4, 3), 7.0, device="cuda")
    ops.llama2_matmul(torch.empty((4, 0), device="cuda"), torch.empty((0, 3), device="cuda"), out=out)
    torch.cuda.synchronize()
    assert (out == 0).all()
    ops.llama2_matmul(torch.empty((0, 5), device="cuda"), torch.ones(5, device="cuda"))


@pytest.mark.parametrize("rows,K", [((288, 288, 288), 288), ((4096, 1024, 1024), 4096), ((11008, 11008), 4096),
                                    ((64, 0, 32), 64), ((17,), 13)])
def test_llama2_matvec_batch_matches_oracle(oracle, rows, K):
    rng = np.random.default_rng(sum(rows) + K)
    ws = [rng.standard_normal((r, K), dtype=np.float32) * np.float32(K ** -0.5) for r in rows]
    x = rng.standard_normal(K, dtype=np.float32)
    outs = ops.llama2_matvec_batch([torch.from_numpy(w).cuda() for w in ws], torch.from_numpy(x).cuda())
    torch.cuda.synchronize()
    for w, o in zip(ws, outs):
        ref = oracle.llama2_matmul(w, x.reshape(K, 1), w.shape[0], 1, K)[:, 0]
        assert (np.abs(o.cpu().numpy() - ref) <= bound(w, x.reshape(K, 1), K)[:, 0]).all()


def _model(tmp_path):
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import make_llama2_model as mk
    return mk.write_model(str(tmp_path), "tiny", seed=0)


def _logits(exe, ckpt, v, out):
    env = dict(os.environ, AKILI_OP="llama2_matmul")
    r = subprocess.run([exe, ckpt, str(v), str(out), *map(str, TOKENS)], capture_output=True, text=True,
                       timeout=300, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    return np.fromfile(out, np.float32).reshape(len(TOKENS), -1)


@pytest.mark.parametrize("exe", ["llama2_logits", "llama2_logits_vxmath"])
def test_reference_llama_forward_on_b200(tmp_path, exe):
    ckpt, _ = _model(tmp_path)
    cpu = _logits(os.path.join(REF, "pin", "llama2_logits"), ckpt, 0, tmp_path / "cpu.bin")
    gpu = _logits(os.path.join(REF, "b200", exe), ckpt, 1, tmp_path / "gpu.bin")
    assert np.abs(gpu - cpu).max() <= 1e-4 * np.abs(cpu).max()
    srt = np.sort(cpu, axis=1)
    clear = (srt[:, -1] - srt[:, -2]) > 1e-3
    assert (gpu.argmax(1) == cpu.argmax(1))[clear].all()


def test_reference_llama_generates_the_cpu_text_on_b200(tmp_path):
    ckpt, tok = _model(tmp_path)
    env = dict(os.environ, AKILI_OP="llama2_matmul")

    def run(exe, v):
        r = subprocess.run([exe, ckpt, "-z", tok, "-t", "0", "-n", "48", "-i", "the cat", "-v", str(v)],
                           capture_output=True, text=True, timeout=300, env=env)
        assert r.returncode == 0, r.stdout + r.stderr
        return r.stdout.replace(">> Using vortex acceleration\n", "").replace("open device connection\n", "")

    cpu = run(os.path.join(REF, "pin", "llama"), 0)
    assert cpu.startswith("the cat")
    assert run(os.path.join(REF, "b200", "llama"), 1) == cpu
    assert run(os.path.join(REF, "b200", "llama_vxmath"), 1) == cpu


@pytest.mark.parametrize("graph", [False, True])
def test_dependent_matvec_chain_sees_each_previous_product(oracle, graph):
    """The matrix-vector kernels launch as programmatic dependents: each may be
    dispatched before the previous kernel of its stream ends, and must wait
    for it before reading its input.  A chain y_{i+1} = W_i . y_i of eight
    launches on one stream (a long one first, then short ones, so that a
    launch that did not wait would read a stale or half-written y_i), run
    directly and replayed from a CUDA graph; each step is checked against the
    oracle applied to the previous step's device output."""
    rng = np.random.default_rng(41)
    dims = [4096, 1024, 1024, 512, 1024, 256, 1024, 512, 768]
    ws = [(rng.standard_normal((dims[i + 1], dims[i])) * dims[i] ** -0.5).astype(np.float32)
          for i in range(len(dims) - 1)]
    big = (rng.standard_normal((8192, dims[0])) * dims[0] ** -0.5).astype(np.float32)
    x = rng.standard_normal(dims[0]).astype(np.float32)
    dw = [torch.from_numpy(w).cuda() for w in ws]
    dbig = torch.from_numpy(big).cuda()
    dx = torch.from_numpy(x).cuda()
    ys = [torch.empty(d, device="cuda", dtype=torch.float32) for d in dims[1:]]
    scratch = torch.empty(big.shape[0], device="cuda", dtype=torch.float32)

    def chain(stream):
        ops.llama2_matmul(dbig, dx, out=scratch, stream=stream)  # a long launch ahead of the chain
        prev = dx
        for w, y in zip(dw, ys):
            ops.llama2_matmul(w, prev, out=y, stream=stream)
            prev = y

    stream = torch.cuda.Stream()
    torch.cuda.synchronize()
    if graph:
        with torch.cuda.stream(stream):
            chain(stream)  # warm-up outside the capture
        torch.cuda.synchronize()
        for y in ys:
            y.fill_(float("nan"))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            chain(stream)
        g.replay()
    else:
        with torch.cuda.stream(stream):
            chain(stream)
    torch.cuda.synchronize()
    assert ops.device_status() == 0
    prev = x
    for i, (w, y) in enumerate(zip(ws, ys)):
        got = y.cpu().numpy()
        ref = oracle.llama2_matmul(w, prev.reshape(-1, 1), w.shape[0], 1, w.shape[1])[:, 0]
        err = np.abs(got.astype(np.float64) - ref)
        assert (err <= bound(w, prev.reshape(-1, 1), w.shape[1])[:, 0]).all(), f"step {i}: max err {err.max():.3e}"
        prev = got
