"""Device-side failure detection without a GPU fault.

Every mbarrier wait in the kernels is bounded; on expiry the kernel records
the wait site in the device status word and returns, so the context stays
usable.  akili_selftest_wait_timeout launches one CTA whose wait can never
complete (an mbarrier nothing arrives at) with a short limit: the status word
must report it, clearing must reset it, and the next op must run correctly.
"""
import ctypes as C

import numpy as np
import pytest

torch = pytest.importorskip("torch")

from akili_bench_b200 import abi, ops  # noqa: E402
from akili_bench_b200.parity import assert_parity  # noqa: E402

pytestmark = pytest.mark.gpu


def test_wait_that_never_completes_is_reported_and_context_survives(oracle):
    ops.device_status(clear=True)
    ops.selftest_wait_timeout(20000)  # 20 ms
    # the C entry returns AKILI_E_DEVICE_TIMEOUT and the code of the wait
    v = C.c_uint32(0)
    assert abi.load().akili_device_status(C.byref(v), 0) == abi.E_DEVICE_TIMEOUT
    assert v.value == ops.STATUS_SELFTEST
    assert ops.device_status(clear=True) == ops.STATUS_SELFTEST
    assert ops.device_status(clear=True) == 0

    # the context is still usable: a GEMM afterwards is correct and clean
    rng = np.random.default_rng(5)
    M, N, K = 256, 264, 136
    x = rng.standard_normal((M, K), dtype=np.float32).astype(np.float16).astype(np.float32)
    w = rng.standard_normal((K, N), dtype=np.float32).astype(np.float16).astype(np.float32)
    b = rng.standard_normal(N, dtype=np.float32)
    got = ops.kbt_gemm_add_relu(torch.from_numpy(x).cuda().half(), torch.from_numpy(w).cuda().half(),
                            torch.from_numpy(b).cuda(), out_dtype=torch.float32).cpu().numpy()
    assert ops.device_status() == 0
    assert_parity(got, oracle.kbt_gemm_add_relu(x, w, b, M, N, K), what="add_relu after a timed-out wait")


@pytest.mark.parametrize("limit_us", [0, 1000001])
def test_selftest_limit_is_validated(limit_us):
    with pytest.raises(abi.AkiliError):
        ops.selftest_wait_timeout(limit_us)
