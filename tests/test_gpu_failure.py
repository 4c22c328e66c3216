"""Failure detection on the device without a GPU fault.

Every mbarrier wait of the tcgen05 kernels is bounded: when it runs out the
kernel records a code in the stream's error word, stops its roles and
returns, and remora_b200_synchronize reports REMORA_ERR_TIMEOUT (the
reference surfaces device errors as CUDAError, remora/runtime.py:477-491).
remora_b200_wait_check runs that same wait on a barrier nothing completes,
with a short limit, so the timeout path is exercised with nothing in flight.
After it the context and the device keep working."""

from __future__ import annotations

import numpy as np
import pytest

from conftest import to_dev, to_host
from remora_b200 import ops
from remora_b200.errors import RemoraTimeoutError

pytestmark = pytest.mark.gpu

LIMIT = 20_000_000  # SM clock cycles, about 10 ms


def test_a_wait_that_runs_out_reports_timeout_and_the_device_keeps_working(cuda):
    ops.synchronize(cuda.index)  # nothing pending
    ops.wait_check(LIMIT, signal=False, device=cuda.index)
    with pytest.raises(RemoraTimeoutError):
        ops.synchronize(cuda.index)
    # the error word was cleared by the report; the next check is clean
    ops.synchronize(cuda.index)
    # and the device still computes: a GEMM on the tensor cores (whose own
    # waits share the error word) and a fold
    a = np.random.default_rng(0).uniform(-1, 1, (256, 128)).astype(np.float32)
    b = np.random.default_rng(1).uniform(-1, 1, (128, 192)).astype(np.float32)
    got = to_host(ops.gemm(to_dev(a, cuda), to_dev(b, cuda), precision="3xtf32"))
    np.testing.assert_allclose(got, a.astype(np.float64) @ b, rtol=1e-4, atol=1e-4)
    s = to_host(ops.fold(to_dev(a, cuda), mode="all"))
    assert abs(float(s) - float(a.astype(np.float64).sum())) < 1e-2


def test_a_signalled_wait_completes_without_error(cuda):
    ops.synchronize(cuda.index)
    ops.wait_check(LIMIT, signal=True, device=cuda.index)
    ops.synchronize(cuda.index)


def test_wait_check_rejects_a_limit_out_of_range(cuda):
    from remora_b200.errors import RemoraB200Error

    with pytest.raises(RemoraB200Error):
        ops.wait_check(-1, device=cuda.index)
    with pytest.raises(RemoraB200Error):
        ops.wait_check(1 << 41, device=cuda.index)
