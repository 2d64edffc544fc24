"""GPU: the failure paths of the build, exercised without faulting or hanging
the GPU.

The reference's only failure handling is decline-then-fallback
(zblas/zblas_gpu.cpp:184-201).  Here every device-side wait is bounded:

  - zlift_wait_probe launches a kernel whose mbarrier wait nothing completes;
    with a 1 ms limit it returns on its own, zlift_device_error() reports
    error 1 once (then 0), and the context keeps working (a GEMM right after
    matches the oracle);
  - zlift_set_wait_limit_ns sets the limit every kernel of the library uses,
    and ordinary calls still pass with a short one;
  - zlift_part_comm_wait gives up at its deadline and aborts the NCCL
    communicator when the stream it watches does not finish in time (here a
    stream held by a 300 ms bounded wait, on a one-rank communicator).
"""
import time

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _small_gemm_ok(h, oracle_lib):
    from tests.helpers import as_float, from_dev, normwise, to_dev
    from zlift_b200 import inputs
    m = n = k = 256
    A = inputs.make("bf16", "normal", 1, m * k)
    B = inputs.make("bf16", "normal", 2, k * n)
    want = np.zeros(m * n, np.uint16)
    assert oracle_lib.gemm_ex(0, 0, m, n, k, 1.0, A, 14, m, B, 14, k, 0.0, want, 14, m) == 0
    dA, dB = to_dev(A, "bf16"), to_dev(B, "bf16")
    dC = to_dev(np.zeros(m * n, np.uint16), "bf16")
    assert h.gemm_ex(0, 0, m, n, k, 1.0, dA, 14, m, dB, 14, k, 0.0, dC, 14, m) == 0
    return normwise(as_float(from_dev(dC, "bf16"), "bf16"), as_float(want, "bf16")) <= 1e-2


def test_bounded_wait_reports_and_returns(cuda, oracle_lib):
    import torch
    from zlift_b200 import Handle, blas, load
    lib = load()
    assert blas.device_error() == 0
    s = torch.cuda.Stream()
    t0 = time.perf_counter()
    assert lib.zlift_wait_probe(1_000_000, s.cuda_stream) == 0      # 1 ms limit
    s.synchronize()
    dt = time.perf_counter() - t0
    assert 1e-3 <= dt < 5.0, dt
    assert blas.device_error() == 1          # kErrWaitTimeout, read and cleared
    assert blas.device_error() == 0
    with Handle() as h:
        assert _small_gemm_ok(h, oracle_lib)
    assert blas.device_error() == 0


def test_wait_probe_rejects_bad_limits(cuda):
    from zlift_b200 import load
    lib = load()
    assert lib.zlift_wait_probe(0, None) == 7
    assert lib.zlift_wait_probe(20_000_000_000, None) == 7


def test_wait_limit_is_settable(cuda, oracle_lib):
    from zlift_b200 import Handle, blas, load
    lib = load()
    default = lib.zlift_get_wait_limit_ns()
    assert default == 2_000_000_000
    assert lib.zlift_set_wait_limit_ns(0) == 7
    try:
        assert lib.zlift_set_wait_limit_ns(50_000_000) == 0       # 50 ms
        assert lib.zlift_get_wait_limit_ns() == 50_000_000
        with Handle() as h:
            assert _small_gemm_ok(h, oracle_lib)
        assert blas.device_error() == 0
    finally:
        assert lib.zlift_set_wait_limit_ns(default) == 0
    assert lib.zlift_get_wait_limit_ns() == default


def test_comm_wait_deadline_aborts(cuda):
    """zlift_part_comm_wait: a stream that outlives the deadline gives 200
    and an aborted communicator; nothing is left running on the GPU."""
    import torch
    from zlift_b200 import blas, load, partition
    lib = load()
    comm = partition.Comm(1, 0, partition.Comm.unique_id())
    s = torch.cuda.Stream()
    assert lib.zlift_wait_probe(300_000_000, s.cuda_stream) == 0    # holds s for 300 ms
    t0 = time.perf_counter()
    rc = comm.wait(s, timeout_ms=20)
    dt = time.perf_counter() - t0
    assert rc == 200, rc
    # the deadline is checked every 0.2 ms; ncclCommAbort itself then takes
    # a few seconds (it tears down NCCL's proxy threads)
    assert dt < 30.0, dt
    assert comm.c is None                  # aborted by the library, dropped here
    s.synchronize()                        # the probe ends by itself
    assert blas.device_error() == 1
    # a fresh communicator works: the stream is idle, so the wait returns 0
    comm2 = partition.Comm(1, 0, partition.Comm.unique_id())
    try:
        assert comm2.wait(s, timeout_ms=1000) == 0
    finally:
        comm2.close()
