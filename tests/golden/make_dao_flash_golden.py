"""Golden vectors of akili-bench's causal flash CPU gold (attention_cpu).

Run here, where the reference tree exists:
    python oracle/build_oracle.py              # builds oracle/_ref/libdao_flash_ref.so
    python tests/golden/make_dao_flash_golden.py

``benchmarks/cupbop_dao_flash/dao_flash_cupbop.cu`` ships no fixtures: its
test (``run_test``, ``:171-244``) fills Q, K and V from ``srand(seed)`` /
``rand() % 100 / 100.0f - 0.5f`` (interleaved per element, ``:188-193``) and
compares its kernel with its CPU gold ``attention_cpu`` (``:134-169``: scale
1/sqrt(d), key j > query i scored -1e30f, N <= 64).  This script calls that
gold, built unchanged from the reference source, on

* the reference's own test configurations (``main``, ``:248-265``) with
  the same seeds and fill order (glibc ``rand`` through ctypes), and
* larger heads within its N <= 64 limit, with seeded N(0,1) inputs,

and writes ``dao_flash__<name>.npz`` holding q, k, v [B, nh, N, d], the
reference output ``expected`` and the case's ``causal`` flag.
"""
from __future__ import annotations

import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
LIB = os.path.join(ROOT, "oracle", "_ref", "libdao_flash_ref.so")

# (name, B, nh, N, d, causal, seed): the reference's run_test calls (dao_flash_cupbop.cu:252-265)
REFERENCE_CASES = [
    ("noncausal_single", 1, 1, 8, 8, 0, 42),
    ("noncausal_multi_tile", 1, 1, 16, 4, 0, 123),
    ("noncausal_multi_head", 1, 2, 8, 4, 0, 456),
    ("causal_single", 1, 1, 8, 8, 1, 42),
    ("causal_multi_tile", 1, 1, 16, 4, 1, 123),
    ("causal_multi_head", 1, 2, 8, 4, 1, 456),
]
# wider heads inside the gold's N <= 64 bound, N(0,1) inputs from numpy seeds
NORMAL_CASES = [
    ("n64d64_causal", 1, 2, 64, 64, 1, 7),
    ("n64d128_causal", 2, 1, 64, 128, 1, 8),
    ("n40d16_causal", 1, 1, 40, 16, 1, 9),
    ("n64d64_noncausal", 1, 1, 64, 64, 0, 10),
]


def glibc_inputs(B, nh, N, d, seed):
    """run_test's fill (dao_flash_cupbop.cu:188-193), element by element."""
    libc = C.CDLL("libc.so.6")
    libc.srand(C.c_uint(seed))
    n = B * nh * N * d
    vals = np.empty((n, 3), np.float32)
    for i in range(n):
        for j in range(3):
            vals[i, j] = np.float32(libc.rand() % 100) / np.float32(100.0) - np.float32(0.5)
    return [vals[:, j].reshape(B, nh, N, d).copy() for j in range(3)]


def reference_attention(lib, q, k, v, causal):
    B, nh, N, d = q.shape
    o = np.zeros_like(q)
    f = lambda a: a.ctypes.data_as(C.POINTER(C.c_float))  # noqa: E731
    rc = lib.akili_ref_attention_cpu(f(q), f(k), f(v), f(o), B, nh, N, d, causal)
    assert rc == 0
    return o


def main() -> int:
    if not os.path.exists(LIB):
        print(f"{LIB} missing: run python oracle/build_oracle.py first", file=sys.stderr)
        return 1
    lib = C.CDLL(LIB)
    for name, B, nh, N, d, causal, seed in REFERENCE_CASES + NORMAL_CASES:
        if (name, B, nh, N, d, causal, seed) in REFERENCE_CASES:
            q, k, v = glibc_inputs(B, nh, N, d, seed)
        else:
            rng = np.random.default_rng(seed)
            q, k, v = (rng.standard_normal((B, nh, N, d), dtype=np.float32) for _ in range(3))
        o = reference_attention(lib, q, k, v, causal)
        path = os.path.join(HERE, f"dao_flash__{name}.npz")
        np.savez_compressed(path, q=q, k=k, v=v, expected=o, causal=np.int32(causal))
        print(path)
    return 0


if __name__ == "__main__":
    sys.exit(main())
