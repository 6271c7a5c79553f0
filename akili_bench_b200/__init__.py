"""akili_bench_b200 — B200 (sm_100a) backend for akili-bench's kbt_* fused ops and flash forward."""
from . import abi  # noqa: F401

__all__ = ["abi"]
