"""zlift_sgemm_noalloc: the fp32 GEMM for callers that cannot allocate
device memory (graph captures that may not allocate, fully reserved
memory pools, interposition layers that must not change a program's
allocations).  It must give the same results as cublasSgemm_v2, which
allocates its split planes per handle, and as the oracle (the C
restatement of the reference's cblas_sgemm path, zblas/zblas.c:111-130),
while using only the library's fixed 16 MiB device array -- so repeated
calls leave the device's free memory where it was.

Called through the C ABI of libcublas.so.13.  Collected last (file name)
so that a run stopping at the first failure has already run every other
test; it also passes on its own in a fresh process.
"""
import ctypes

import numpy as np
import pytest

from tests.helpers import from_dev, normwise, to_dev

pytestmark = pytest.mark.gpu

TOL = 1e-5          # the fp32 tolerance of the other GEMM tests


def _noalloc(h, ta, tb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc):
    lib = h.lib
    al, be = ctypes.c_float(alpha), ctypes.c_float(beta)
    return lib.zlift_sgemm_noalloc(h.h, ta, tb, m, n, k, ctypes.byref(al), A.data_ptr(), lda,
                                   B.data_ptr(), ldb, ctypes.byref(be), C.data_ptr(), ldc)


@pytest.fixture(scope="module")
def handle(cuda):
    from zlift_b200 import Handle
    with Handle() as h:
        yield h


@pytest.mark.parametrize("ta,tb,m,n,k,alpha,beta", [
    (0, 0, 1024, 1024, 1024, 1.0, 0.0),     # fills the 16 MiB array exactly
    (1, 1, 300, 260, 200, 0.5, -1.5),
    (0, 1, 129, 77, 65, 2.0, 1.0),
])
def test_noalloc_matches_sgemm_twice(handle, oracle_lib, ta, tb, m, n, k, alpha, beta):
    import torch
    from zlift_b200 import inputs
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    for call in range(2):                     # two calls in a row
        hA = inputs.make("f32", "uniform", 10 * call + 1, ar * ac)
        hB = inputs.make("f32", "uniform", 10 * call + 2, br * bc)
        A, B = to_dev(hA, "f32"), to_dev(hB, "f32")
        C0 = inputs.make("f32", "uniform", 10 * call + 3, m * n)
        C_ref, C_new = to_dev(C0, "f32"), to_dev(C0, "f32")
        assert handle.sgemm(ta, tb, m, n, k, alpha, A, ar, B, br, beta, C_ref, m) == 0
        assert _noalloc(handle, ta, tb, m, n, k, alpha, A, ar, B, br, beta, C_new, m) == 0
        torch.cuda.synchronize()
        want = from_dev(C_ref, "f32").astype(np.float64)
        got = from_dev(C_new, "f32").astype(np.float64)
        assert normwise(got, want) <= TOL
        oref = C0.copy()
        assert oracle_lib.gemm_ex(ta, tb, m, n, k, alpha, hA, 0, ar, hB, 0, br, beta, oref, 0,
                                  m) == 0
        assert normwise(got, oref.astype(np.float64)) <= TOL


def test_noalloc_leaves_free_memory_unchanged(handle):
    """After a first call, further calls take no device memory: the free
    memory the driver reports does not move."""
    import torch
    from zlift_b200 import inputs
    m = n = k = 512
    A = to_dev(inputs.make("f32", "uniform", 41, m * k), "f32")
    B = to_dev(inputs.make("f32", "uniform", 42, k * n), "f32")
    C = to_dev(np.zeros(m * n, np.float32), "f32")
    assert _noalloc(handle, 0, 0, m, n, k, 1.0, A, m, B, k, 0.0, C, m) == 0
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    for _ in range(5):
        assert _noalloc(handle, 0, 0, m, n, k, 1.0, A, m, B, k, 0.0, C, m) == 0
    torch.cuda.synchronize()
    free1, _ = torch.cuda.mem_get_info()
    assert free1 == free0


def test_noalloc_rejects_oversize(handle):
    """Beyond the fixed array: CUBLAS_STATUS_INVALID_VALUE, nothing launched."""
    import torch
    from zlift_b200 import blas
    A = torch.zeros(1, dtype=torch.float32, device="cuda")
    n0 = blas.launch_count()
    # 2048 x 2048 x 2048 needs 64 MiB of planes (> 16 MiB); the sizes are
    # rejected before any operand is touched
    assert _noalloc(handle, 0, 0, 2048, 2048, 2048, 1.0, A, 2048, A, 2048, 0.0, A, 2048) == 7
    # sizes whose plane sizes would overflow 64-bit arithmetic if multiplied
    # out unchecked are rejected too
    big = 2 ** 31 - 1
    assert _noalloc(handle, 0, 0, 2 ** 29, 2 ** 29, big, 1.0, A, 2 ** 29, A, big, 0.0, A,
                    2 ** 29) == 7
    assert blas.launch_count() == n0
