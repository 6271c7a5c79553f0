"""The host-side caches of device memory: what keys them, and when they are
dropped.

* libakili's internal scratch is one grow-only buffer per (CUDA context,
  stream).  cudaStreamPerThread is one handle for a different stream in each
  host thread, so for it the calling thread is part of the key.  Two host
  threads on the per-thread stream, each running kbt_gemm_layernorm (two-pass
  form, whose row statistics live in that scratch) on its own shapes at the
  same time, must each match the oracle.
* libakili_vxmath keeps a weight matrix in read-only host memory resident in
  HBM, keyed by its host address.  When that mapping is replaced by another at
  the same address (another file, then writable memory whose bytes change
  between calls), every call must use the bytes mapped at that moment.
"""
import ctypes as C
import os
import threading

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu

HERE = os.path.dirname(os.path.abspath(__file__))
VXMATH = os.path.join(os.path.dirname(HERE), "akili_bench_b200", "libakili_vxmath.so")
CUDA_STREAM_PER_THREAD = 0x2


def test_per_thread_stream_scratch_is_not_shared_between_threads(oracle, monkeypatch):
    monkeypatch.setenv("AKILI_ROWNORM", "0")  # the two-pass form keeps its statistics in the scratch
    shapes = [(520, 4104, 136), (1032, 2056, 264)]
    cases = []
    for t, (M, N, K) in enumerate(shapes):
        rng = np.random.default_rng(101 + t)
        x = rng.standard_normal((M, K)).astype(np.float16)
        w = (rng.standard_normal((K, N)) * K ** -0.5).astype(np.float16)
        b = (rng.standard_normal(N) * 0.02).astype(np.float32)
        g = (1 + rng.standard_normal(N) * 0.02).astype(np.float32)
        beta = (rng.standard_normal(N) * 0.02).astype(np.float32)
        ref = oracle.kbt_gemm_layernorm(x.astype(np.float32), w.astype(np.float32), b, g, beta, M, N, K, 1e-5,
                                        threads=8)
        dev = [torch.from_numpy(a).cuda() for a in (x, w, b, g, beta)]
        out = torch.empty((M, N), dtype=torch.float16, device="cuda")
        cases.append((dev, out, ref))
    torch.cuda.synchronize()
    stream = torch.cuda.ExternalStream(CUDA_STREAM_PER_THREAD)
    errors = []

    def run(case):
        dev, out, _ = case
        try:
            for _ in range(20):
                ops.kbt_gemm_layernorm(*dev, 1e-5, out=out, stream=stream)
        except Exception as e:  # reported on the main thread
            errors.append(e)

    threads = [threading.Thread(target=run, args=(c,)) for c in cases]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    torch.cuda.synchronize()
    assert not errors, errors
    assert ops.device_status() == 0
    for i, (_, out, ref) in enumerate(cases):
        assert_parity(out.float().cpu().numpy(), ref, what=f"per-thread stream, thread {i}")


def _libc():
    libc = C.CDLL("libc.so.6", use_errno=True)
    libc.mmap.restype = C.c_void_p
    libc.mmap.argtypes = [C.c_void_p, C.c_size_t, C.c_int, C.c_int, C.c_int, C.c_long]
    libc.munmap.argtypes = [C.c_void_p, C.c_size_t]
    return libc


PROT_READ, PROT_WRITE = 1, 2
MAP_PRIVATE, MAP_FIXED, MAP_ANONYMOUS = 0x02, 0x10, 0x20
MAP_FAILED = C.c_void_p(-1).value


def test_resident_weights_follow_a_replaced_mapping(oracle, tmp_path):
    if not os.path.exists(VXMATH):
        pytest.fail(f"{VXMATH} is not built")
    M, K = 192, 288
    rng = np.random.default_rng(7)
    mats = [(rng.standard_normal((M, K)) * K ** -0.5).astype(np.float32) for _ in range(3)]
    x = rng.standard_normal(K).astype(np.float32)
    nbytes = mats[0].nbytes
    libc = _libc()
    # benchmarks/llama2/vxmath.h declares these with C++ linkage
    vx = C.CDLL(VXMATH)
    vx_init, vx_matmul, cleanup = vx._Z7vx_initv, vx._Z9vx_matmulPfS_S_iii, vx._Z14matmul_cleanupv
    vx_matmul.argtypes = [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int]
    vx_init()
    c = np.zeros(M, np.float32)

    def product(addr):
        vx_matmul(c.ctypes.data, addr, x.ctypes.data, M, 1, K)
        return c.copy()

    def check(addr, a, what):
        ref = oracle.llama2_matmul(a, x.reshape(K, 1), M, 1, K)[:, 0]
        got = product(addr)
        bound = 4e-6 * K ** 0.5 * (np.abs(a).astype(np.float64) @ np.abs(x).astype(np.float64)) + 1e-30
        assert (np.abs(got - ref) <= bound).all(), what

    fds, addr = [], None
    try:
        for i in range(2):
            p = tmp_path / f"w{i}.bin"
            p.write_bytes(mats[i].tobytes())
            fds.append(os.open(p, os.O_RDONLY))
        # file 0, read-only: uploaded once and resident
        addr = libc.mmap(None, nbytes, PROT_READ, MAP_PRIVATE, fds[0], 0)
        assert addr not in (None, MAP_FAILED)
        check(addr, mats[0], "first mapping")
        check(addr, mats[0], "first mapping, resident")
        # file 1 mapped read-only at the same address
        got = libc.mmap(addr, nbytes, PROT_READ, MAP_PRIVATE | MAP_FIXED, fds[1], 0)
        assert got == addr
        check(addr, mats[1], "second file at the same address")
        # writable memory at the same address, then changed between calls
        got = libc.mmap(addr, nbytes, PROT_READ | PROT_WRITE, MAP_PRIVATE | MAP_FIXED | MAP_ANONYMOUS, -1, 0)
        assert got == addr
        view = np.ctypeslib.as_array((C.c_float * (M * K)).from_address(addr)).reshape(M, K)
        view[:] = mats[2]
        check(addr, mats[2], "writable memory at the same address")
        view[: M // 2] *= np.float32(-1.0)
        changed = view.copy()
        check(addr, changed, "writable memory changed in place")
    finally:
        cleanup()
        if addr not in (None, MAP_FAILED):
            libc.munmap(addr, nbytes)
        for fd in fds:
            os.close(fd)
