"""GEMM parity on the GPU: every case runs through the C ABI of
libcublas.so.13 and is compared with the oracle (a C restatement of
zblas/zblas.c's CPU path) on the same seeded inputs.

Tolerances (normwise, max|x - ref| / max|ref|), from the task statement:
  fp16 / bf16 inputs          <= 1e-2
  fp32 (TF32 math off)        <= 1e-5
  int8 -> int32               bit-exact
Every output buffer carries trailing canary elements that must come back
untouched (bounds check without compute-sanitizer).
"""
import numpy as np
import pytest

from tests.helpers import CUDA_T, as_float, from_dev, normwise, to_dev

pytestmark = pytest.mark.gpu

TOL = {"f16": 1e-2, "bf16": 1e-2, "f32": 1e-5}
CANARY = 64


def _operand(kind, dist, seed, rows, cols, ld, scale=1.0):
    from zlift_b200 import inputs
    n = ld * (cols - 1) + rows if cols > 0 else 0
    return inputs.make(kind, dist, seed, max(n, 1), scale)


def run_gemm(h, oracle, kind, ckind, ta, tb, m, n, k, alpha, beta, lda=None, ldb=None,
             ldc=None, seed=1, dist="normal", scale=1.0):
    from zlift_b200 import blas
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    lda = lda or max(ar, 1)
    ldb = ldb or max(br, 1)
    ldc = ldc or max(m, 1)
    A = _operand(kind, dist, seed, ar, ac, lda, scale)
    B = _operand(kind, dist, seed + 1, br, bc, ldb, scale)
    if ckind == "i32":
        C0 = (np.arange(ldc * n, dtype=np.int64) % 1000 - 500).astype(np.int32)
    else:
        C0 = _operand(ckind, "normal", seed + 2, m, n, ldc)
        if C0.size < max(ldc * n, 1):
            C0 = np.resize(C0, max(ldc * n, 1))
    C0 = C0[: max(ldc * n, 1)].copy()
    compute = blas.COMPUTE_32I if kind == "i8" else blas.COMPUTE_32F

    cref = C0.copy()
    rc = oracle.gemm_ex(ta, tb, m, n, k, alpha, A, CUDA_T[kind], lda, B, CUDA_T[kind], ldb,
                        beta, cref, CUDA_T[ckind], ldc, compute)
    assert rc == 0

    dA, dB = to_dev(A, kind), to_dev(B, kind)
    canary_val = 0x5A5A if ckind in ("f16", "bf16") else 12345
    dC = to_dev(C0, ckind, pad=CANARY, fill=canary_val if ckind != "f32" else 0)
    if ckind == "f32":
        dC[-CANARY:] = 12345.0
    if kind == "f32":
        st = h.sgemm(ta, tb, m, n, k, alpha, dA, lda, dB, ldb, beta, dC, ldc)
    else:
        st = h.gemm_ex(ta, tb, m, n, k, alpha, dA, CUDA_T[kind], lda, dB, CUDA_T[kind], ldb,
                       beta, dC, CUDA_T[ckind], ldc, compute)
    assert st == 0, f"status {st}"
    out = from_dev(dC, ckind)
    assert blas.device_error() == 0
    tail = out[-CANARY:]
    if ckind == "f32":
        assert np.all(tail == np.float32(12345.0)), "wrote past the end of C"
    elif ckind == "i32":
        assert np.all(tail == 12345), "wrote past the end of C"
    else:
        assert np.all(tail == canary_val), "wrote past the end of C"
    out = out[:-CANARY]
    if ckind == "i32":
        np.testing.assert_array_equal(out, cref)
        return 0.0
    # only compare the m x n window (rows >= m inside ldc are untouched padding)
    got = as_float(out, ckind).reshape(n, ldc)[:, :m] if n > 0 else out
    want = as_float(cref, ckind).reshape(n, ldc)[:, :m] if n > 0 else cref
    pad_got = as_float(out, ckind).reshape(n, ldc)[:, m:]
    pad_want = as_float(C0, ckind).reshape(n, ldc)[:, m:]
    np.testing.assert_array_equal(pad_got, pad_want)
    err = normwise(got, want)
    assert err <= TOL[kind], f"normwise error {err:.3e}"
    return err


@pytest.fixture(scope="module")
def handle(cuda):
    from zlift_b200 import Handle
    with Handle() as h:
        yield h


SHAPES = [
    (1, 1, 1), (7, 5, 3), (64, 64, 64), (128, 256, 64), (129, 257, 65), (256, 512, 128),
    (300, 200, 136), (1000, 700, 520), (512, 512, 512),
]


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_gemm_ex_16bit(handle, oracle_lib, kind, ta, tb, m, n, k):
    run_gemm(handle, oracle_lib, kind, kind, ta, tb, m, n, k, 1.0, 0.0, seed=m + n + k)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
@pytest.mark.parametrize("m,n,k", [(256, 384, 192), (100, 300, 72)])
def test_gemm_ex_alpha_beta_f32_out(handle, oracle_lib, kind, m, n, k):
    run_gemm(handle, oracle_lib, kind, kind, 0, 1, m, n, k, 0.75, 0.5)
    run_gemm(handle, oracle_lib, kind, "f32", 1, 0, m, n, k, -1.25, 2.0)


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (33, 17, 9), (128, 128, 128), (300, 260, 200),
                                   (1024, 1024, 1024)])
def test_sgemm(handle, oracle_lib, ta, tb, m, n, k):
    run_gemm(handle, oracle_lib, "f32", "f32", ta, tb, m, n, k, 1.0, 0.0, dist="uniform")


def test_sgemm_alpha_beta(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "f32", "f32", 0, 0, 200, 150, 300, 0.5, -1.5, dist="uniform")


@pytest.mark.parametrize("ta,tb", [(0, 0), (0, 1), (1, 0), (1, 1)])
@pytest.mark.parametrize("m,n,k", [(1, 1, 1), (64, 48, 40), (128, 256, 128), (300, 260, 200),
                                   (512, 384, 1024)])
def test_gemm_ex_int8(handle, oracle_lib, ta, tb, m, n, k):
    run_gemm(handle, oracle_lib, "i8", "i32", ta, tb, m, n, k, 1, 0, dist="int8")


def test_gemm_ex_int8_alpha_beta(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "i8", "i32", 1, 0, 256, 320, 512, 3, -2, dist="int8")


@pytest.mark.parametrize("kind", ["f16", "bf16", "f32", "i8"])
def test_unaligned_leading_dims(handle, oracle_lib, kind):
    """Leading dimensions that are not 16-byte multiples take the general
    kernel; results must still match."""
    ck = {"i8": "i32"}.get(kind, kind)
    dist = "int8" if kind == "i8" else "uniform"
    run_gemm(handle, oracle_lib, kind, ck, 0, 1, 77, 45, 33, 1, 0, lda=79, ldb=47, ldc=81,
             dist=dist)


@pytest.mark.parametrize("kind", ["f16", "bf16"])
def test_padded_leading_dims(handle, oracle_lib, kind):
    run_gemm(handle, oracle_lib, kind, kind, 1, 0, 200, 100, 96, 1.0, 0.5, lda=104, ldb=128,
             ldc=208)


def test_k_zero_scales_c(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "f16", "f16", 0, 0, 64, 32, 0, 1.0, 0.5, lda=64, ldb=1)


def test_device_pointer_mode(handle, oracle_lib, cuda):
    import torch
    from zlift_b200 import blas
    m = n = k = 256
    from zlift_b200 import inputs
    A = inputs.make("bf16", "normal", 9, m * k)
    B = inputs.make("bf16", "normal", 10, k * n)
    dA, dB = to_dev(A, "bf16"), to_dev(B, "bf16")
    dC = torch.zeros(m * n, dtype=torch.float32, device=cuda)
    al = torch.tensor([0.5], dtype=torch.float32, device=cuda)
    be = torch.tensor([0.0], dtype=torch.float32, device=cuda)
    assert handle.set_pointer_mode(blas.POINTER_MODE_DEVICE) == 0
    try:
        st = handle.gemm_ex(0, 0, m, n, k, al, dA, 14, m, dB, 14, k, be, dC, 0, m)
    finally:
        handle.set_pointer_mode(blas.POINTER_MODE_HOST)
    assert st == 0
    cref = np.zeros(m * n, dtype=np.float32)
    oracle_lib.gemm_ex(0, 0, m, n, k, 0.5, A, 14, m, B, 14, k, 0.0, cref, 0, m)
    assert normwise(dC.cpu().numpy().astype(np.float64), cref.astype(np.float64)) < 1e-2


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("ta,tb", [(0, 0), (1, 1)])
def test_strided_batched(handle, oracle_lib, kind, ta, tb):
    from zlift_b200 import blas, inputs
    m, n, k, batch = 96, 160, 72, 5
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    sA, sB, sC = ar * ac + 8, br * bc + 16, m * n + 24
    A = inputs.make(kind, "normal", 1, sA * batch)
    B = inputs.make(kind, "normal", 2, sB * batch)
    C0 = inputs.make(kind, "normal", 3, sC * batch)
    al, be = 1.0 / np.sqrt(k), 0.25
    cref = C0.copy()
    assert oracle_lib.gemm_strided_batched_ex(ta, tb, m, n, k, al, A, CUDA_T[kind], ar, sA, B,
                                              CUDA_T[kind], br, sB, be, cref, CUDA_T[kind], m,
                                              sC, batch) == 0
    dA, dB, dC = to_dev(A, kind), to_dev(B, kind), to_dev(C0, kind)
    st = handle.gemm_strided_batched_ex(ta, tb, m, n, k, al, dA, CUDA_T[kind], ar, sA, dB,
                                        CUDA_T[kind], br, sB, be, dC, CUDA_T[kind], m, sC,
                                        batch)
    assert st == 0
    out = as_float(from_dev(dC, kind), kind).reshape(batch, sC)
    want = as_float(cref, kind).reshape(batch, sC)
    assert normwise(out[:, : m * n], want[:, : m * n]) <= 1e-2
    # the gaps between matrices are never written
    np.testing.assert_array_equal(out[:, m * n:], as_float(C0, kind).reshape(batch, sC)[:, m * n:])


def test_strided_batched_int8(handle, oracle_lib):
    from zlift_b200 import inputs
    m, n, k, batch = 128, 96, 160, 3
    A = inputs.make("i8", "int8", 4, k * m * batch)
    B = inputs.make("i8", "int8", 5, k * n * batch)
    cref = np.zeros(m * n * batch, dtype=np.int32)
    assert oracle_lib.gemm_strided_batched_ex(1, 0, m, n, k, 1, A, 3, k, k * m, B, 3, k, k * n,
                                              0, cref, 10, m, m * n, batch, 72) == 0
    dA, dB = to_dev(A, "i8"), to_dev(B, "i8")
    dC = to_dev(np.zeros(m * n * batch, dtype=np.int32), "i32")
    st = handle.gemm_strided_batched_ex(1, 0, m, n, k, 1, dA, 3, k, k * m, dB, 3, k, k * n, 0,
                                        dC, 10, m, m * n, batch, 72)
    assert st == 0
    np.testing.assert_array_equal(from_dev(dC, "i32"), cref)


def test_repeat_is_deterministic(handle, oracle_lib, cuda):
    """Bitwise-identical outputs across repeats (no race in the pipeline)."""
    import torch
    from zlift_b200 import inputs
    m = n = k = 768
    A = to_dev(inputs.make("f16", "normal", 1, m * k), "f16")
    B = to_dev(inputs.make("f16", "normal", 2, k * n), "f16")
    outs = []
    for _ in range(3):
        C = torch.zeros(m * n, dtype=torch.float16, device=cuda)
        assert handle.gemm_ex(0, 1, m, n, k, 1.0, A, 2, m, B, 2, n, 0.0, C, 2, m) == 0
        outs.append(C.clone())
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])


def test_sgemm_tf32_math_mode(handle, oracle_lib):
    """CUBLAS_TF32_TENSOR_OP_MATH: one tf32 product (about 1e-3 relative)."""
    from zlift_b200 import blas
    assert handle.set_math_mode(blas.TF32_TENSOR_OP_MATH) == 0
    try:
        m, n, k = 256, 192, 320
        from zlift_b200 import inputs
        A = inputs.make("f32", "uniform", 1, m * k)
        B = inputs.make("f32", "uniform", 2, k * n)
        ref = np.zeros(m * n, np.float32)
        oracle_lib.gemm_ex(0, 0, m, n, k, 1.0, A, 0, m, B, 0, k, 0.0, ref, 0, m)
        dA, dB = to_dev(A, "f32"), to_dev(B, "f32")
        dC = to_dev(np.zeros(m * n, np.float32), "f32")
        assert handle.sgemm(0, 0, m, n, k, 1.0, dA, m, dB, k, 0.0, dC, m) == 0
        err = normwise(from_dev(dC, "f32").astype(np.float64), ref.astype(np.float64))
        assert err < 5e-3
    finally:
        handle.set_math_mode(blas.DEFAULT_MATH)


# Shapes large enough for the CTA-pair kernel (256-row tiles split over two
# SMs): >= 148 tiles of 128 x 256 and >= 74 pair tiles.  M = 1200 leaves the
# second CTA of the last pair tile partly past the end of C.
@pytest.mark.parametrize("kind", ["f16", "bf16", "i8"])
@pytest.mark.parametrize("ta,tb", [(0, 1), (1, 0), (0, 0), (1, 1)])
def test_pair_tiles(handle, oracle_lib, kind, ta, tb):
    if kind == "i8":
        run_gemm(handle, oracle_lib, "i8", "i32", ta, tb, 1200, 4000, 2080, 2, -1, dist="int8")
    else:
        run_gemm(handle, oracle_lib, kind, kind, ta, tb, 1200, 4000, 1040, 1.0, 0.5, seed=7)


def test_pair_tiles_f32_out(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "bf16", "f32", 0, 1, 2048, 2560, 1024, 0.5, 0.0, seed=3)


def test_pair_tiles_strided_batched(handle, oracle_lib):
    from zlift_b200 import inputs
    m, n, k, batch = 256, 256, 1024, 150
    A = inputs.make("bf16", "normal", 21, m * k * batch)
    B = inputs.make("bf16", "normal", 22, k * n * batch)
    C0 = np.zeros(m * n * batch, np.uint16)
    cref = C0.copy()
    assert oracle_lib.gemm_strided_batched_ex(0, 0, m, n, k, 0.125, A, 14, m, m * k, B, 14, k,
                                              k * n, 0.0, cref, 14, m, m * n, batch) == 0
    dA, dB, dC = to_dev(A, "bf16"), to_dev(B, "bf16"), to_dev(C0, "bf16")
    assert handle.gemm_strided_batched_ex(0, 0, m, n, k, 0.125, dA, 14, m, m * k, dB, 14, k,
                                          k * n, 0.0, dC, 14, m, m * n, batch) == 0
    got = as_float(from_dev(dC, "bf16"), "bf16")
    assert normwise(got, as_float(cref, "bf16")) <= 1e-2


@pytest.mark.parametrize("k", [1024, 4096, 16384])
def test_sgemm_long_k_accuracy(handle, oracle_lib, k):
    """fp32 GEMM accuracy does not decay with K: the 3xTF32 kernel adds
    128-deep accumulator chunks in fp32 (round to nearest), so the error
    against an fp64 product of the same inputs stays near 1e-6 where one
    tensor-core accumulation over K reached 1.2e-4 at K = 16384."""
    from zlift_b200 import inputs
    m = n = 256
    A = inputs.make("f32", "uniform", 61, m * k)
    B = inputs.make("f32", "uniform", 62, k * n)
    exact = (A.astype(np.float64).reshape(k, m).T @ B.astype(np.float64).reshape(n, k).T)
    exact = exact.T.reshape(-1)
    cref = np.zeros(m * n, np.float32)
    assert oracle_lib.gemm_ex(0, 0, m, n, k, 1.0, A, 0, m, B, 0, k, 0.0, cref, 0, m) == 0
    dA, dB = to_dev(A, "f32"), to_dev(B, "f32")
    dC = to_dev(np.zeros(m * n, np.float32), "f32")
    assert handle.sgemm(0, 0, m, n, k, 1.0, dA, m, dB, k, 0.0, dC, m) == 0
    got = from_dev(dC, "f32").astype(np.float64)
    assert normwise(got, exact) <= 2e-6
    assert normwise(got, cref.astype(np.float64)) <= 1e-5
