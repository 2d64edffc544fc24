"""GPU: the N split of a sparse last wave (half-width units).

When the last wave of a GEMM's tiles fills at most half of the persistent
CTAs (or CTA pairs), each of its tiles runs as two units of half the tile's
columns.  Each output element is still the same dot product accumulated in
the same K order, so the result must be bit-identical to the run without
the split (ZBLAS_TAIL_HALVES=0), and match the oracle.  Shapes are chosen so
that every tile configuration (ZBLAS_GEMM_CFG) ends with a sparse wave.
"""
import os

import numpy as np
import pytest

from tests.helpers import CUDA_T, as_float, from_dev, normwise, to_dev

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def handle(cuda):
    from zlift_b200 import Handle
    with Handle() as h:
        yield h


def _run(handle, kind, ckind, ta, tb, m, n, k, A, B, C0, halves):
    from zlift_b200 import blas
    os.environ["ZBLAS_TAIL_HALVES"] = "1" if halves else "0"
    try:
        ar = m if ta == 0 else k
        br = k if tb == 0 else n
        dA, dB, dC = to_dev(A, kind), to_dev(B, kind), to_dev(C0, ckind)
        compute = blas.COMPUTE_32I if kind == "i8" else blas.COMPUTE_32F
        alpha, beta = (1, 0) if kind == "i8" else (1.0, 0.5)
        assert handle.gemm_ex(ta, tb, m, n, k, alpha, dA, CUDA_T[kind], ar, dB, CUDA_T[kind], br,
                              beta, dC, CUDA_T[ckind], m, compute) == 0
        out = from_dev(dC, ckind)
        assert blas.device_error() == 0
        return out
    finally:
        os.environ.pop("ZBLAS_TAIL_HALVES", None)


@pytest.mark.parametrize("cfg", ["p256", "s256", "s128", "p128"])
@pytest.mark.parametrize("ta,tb", [(0, 1), (1, 0), (0, 0)])
def test_tail_halves_f16(handle, oracle_lib, cfg, ta, tb):
    from zlift_b200 import inputs
    m, n, k = 2560, 4096, 1024
    A = inputs.make("f16", "normal", 71, m * k, 1 / 32)
    B = inputs.make("f16", "normal", 72, k * n, 1 / 32)
    C0 = inputs.make("f16", "normal", 73, m * n)
    os.environ["ZBLAS_GEMM_CFG"] = cfg
    try:
        full = _run(handle, "f16", "f16", ta, tb, m, n, k, A, B, C0, halves=False)
        half = _run(handle, "f16", "f16", ta, tb, m, n, k, A, B, C0, halves=True)
    finally:
        os.environ.pop("ZBLAS_GEMM_CFG", None)
    np.testing.assert_array_equal(half, full)
    want = C0.copy()
    ar = m if ta == 0 else k
    br = k if tb == 0 else n
    assert oracle_lib.gemm_ex(ta, tb, m, n, k, 1.0, A, 2, ar, B, 2, br, 0.5, want, 2, m) == 0
    assert normwise(as_float(half, "f16"), as_float(want, "f16")) <= 1e-2


@pytest.mark.parametrize("cfg", ["p256", "s256"])
def test_tail_halves_int8(handle, oracle_lib, cfg):
    """int8 TN (both operands K-major), bit-exact against the oracle."""
    from zlift_b200 import inputs
    m, n, k = 2560, 4096, 2048
    A = inputs.make("i8", "int8", 81, k * m)
    B = inputs.make("i8", "int8", 82, k * n)
    C0 = np.zeros(m * n, np.int32)
    os.environ["ZBLAS_GEMM_CFG"] = cfg
    try:
        full = _run(handle, "i8", "i32", 1, 0, m, n, k, A, B, C0, halves=False)
        half = _run(handle, "i8", "i32", 1, 0, m, n, k, A, B, C0, halves=True)
    finally:
        os.environ.pop("ZBLAS_GEMM_CFG", None)
    np.testing.assert_array_equal(half, full)
    want = C0.copy()
    assert oracle_lib.gemm_ex(1, 0, m, n, k, 1, A, 3, k, B, 3, k, 0, want, 10, m, 72) == 0
    np.testing.assert_array_equal(half, want)
