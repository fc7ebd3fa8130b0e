"""Failure detection on the device without a fault: a kernel wait that nothing
completes (an mbarrier no thread arrives at) runs through the same bounded
wait every engine kernel uses, gives up after its limit, leaves its code in
the error word and returns; the host sees DTTS_ERR_TIMEOUT and the context
stays usable (a GEMM on the same device afterwards is exact)."""
import time

import numpy as np
import pytest

import dtts
from helpers import bf16, rel

pytestmark = pytest.mark.gpu


def test_device_wait_limit_reports_and_context_survives():
    t0 = time.perf_counter()
    st, code = dtts.selftest_wait_limit()
    dt = time.perf_counter() - t0
    assert st == dtts.ERR_TIMEOUT and code == 1, (st, code)
    assert 1.5 < dt < 30.0    # the 2 s limit, not an endless spin
    rng = np.random.default_rng(0)
    A = rng.standard_normal((256, 512)).astype(np.float32)
    B = rng.standard_normal((256, 512)).astype(np.float32)
    got = dtts.selftest_gemm(A, B)
    want = bf16(A).astype(np.float64) @ bf16(B).astype(np.float64).T
    assert rel(got, want) <= 1e-5
