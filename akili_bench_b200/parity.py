"""Parity helpers shared by the GPU tests, smoke() and bench.py's check.

The parity bar: max|err| <= 1e-2 * max|ref| over the output
and cosine similarity >= 0.9999 per output row (over the whole vector for the
[M]-shaped outputs).  The reference side is the CPU oracle evaluated on the
same fp16-rounded operands the device sees.
"""
from __future__ import annotations

import numpy as np

MAX_ERR_FRAC = 1e-2
MIN_ROW_COS = 0.9999


def parity(got, ref, rows: bool = True) -> dict:
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape, (got.shape, ref.shape)
    if not np.isfinite(got).all():
        return {"ok": False, "why": "non-finite output", "max_err": float("inf"), "min_cos": -1.0}
    err = np.abs(got - ref)
    scale = float(np.abs(ref).max()) if ref.size else 0.0
    max_err = float(err.max()) if err.size else 0.0
    g2 = got.reshape(got.shape[0], -1) if (rows and got.ndim >= 2) else got.reshape(1, -1)
    r2 = ref.reshape(ref.shape[0], -1) if (rows and ref.ndim >= 2) else ref.reshape(1, -1)
    num = (g2 * r2).sum(1)
    den = np.sqrt((g2 * g2).sum(1) * (r2 * r2).sum(1))
    # rows that are (numerically) zero on both sides count as identical
    zero = (np.sqrt((r2 * r2).sum(1)) <= 1e-30) & (np.sqrt((g2 * g2).sum(1)) <= 1e-30)
    cos = np.where(zero, 1.0, num / np.where(den > 0, den, 1.0))
    min_cos = float(cos.min()) if cos.size else 1.0
    ok = max_err <= MAX_ERR_FRAC * scale + 1e-30 and min_cos >= MIN_ROW_COS
    return {"ok": bool(ok), "max_err": max_err, "max_ref": scale, "min_cos": min_cos,
            "err_frac": max_err / scale if scale else 0.0}


def assert_parity(got, ref, rows: bool = True, what: str = "") -> dict:
    p = parity(got, ref, rows)
    assert p["ok"], f"{what}: parity failed {p}"
    return p
