"""GPU parity at the benchmark configurations' exact sizes, through the C ABI
of libcublas.so.13, against the oracle (oracle/zlift_oracle.c) on the same
seeded inputs:

  cublasGemmEx fp16 4096^3, transa=N transb=T, alpha=1 beta=0.5, fp16 C
      (zblas/zblas.c:357-391): every element of C, normwise <= 1e-2;
  cublasGemmStridedBatchedEx bf16, batch 256 of 512^3 NN, alpha=1/sqrt(512)
      beta=0 (zblas/zblas.c:491-511): every batch, normwise <= 1e-2 each;
  cublasGemmEx int8 x int8 -> int32, M=2048 K=4096 N=14336 TN: bit-exact
      over all of C;
  the batched call split into two batch ranges through
      zlift_part_gemm_strided_batched_ex: bit-equal to the one-shot call;
  cublasHgemm, cublasSgemmEx and cublasSgemmStridedBatched against the
      oracle (zblas/zblas.c:278-304, :480-487, :145-168).

The kernel's tile configuration, wave count and K-split decision depend on
the shape, so these sizes are checked as they are benchmarked.  Outputs carry
canary tails that must come back untouched.
"""
import math

import numpy as np
import pytest

from tests.helpers import as_float, from_dev, normwise, to_dev

pytestmark = pytest.mark.gpu

CANARY = 256


@pytest.fixture(scope="module")
def handle(cuda):
    from zlift_b200 import Handle
    with Handle() as h:
        yield h


def _canary_ok(out, kind, value):
    tail = out[-CANARY:]
    return bool(np.all(tail == value))


def test_gemm_ex_f16_4096_nt_beta_full(handle, oracle_lib):
    """cublasGemmEx fp16 4096^3 NT, alpha 1, beta 0.5: all of C vs the oracle."""
    from zlift_b200 import blas, inputs
    M = N = K = 4096
    A = inputs.make("f16", "normal", 101, M * K, 1.0 / 64)     # M x K, lda = M
    B = inputs.make("f16", "normal", 102, N * K, 1.0 / 64)     # op T: stored N x K, ldb = N
    C0 = inputs.make("f16", "normal", 103, M * N)
    want = C0.copy()
    assert oracle_lib.gemm_ex(0, 1, M, N, K, 1.0, A, 2, M, B, 2, N, 0.5, want, 2, M) == 0
    dA, dB = to_dev(A, "f16"), to_dev(B, "f16")
    dC = to_dev(C0, "f16", pad=CANARY, fill=0x5A5A)
    assert handle.gemm_ex(0, 1, M, N, K, 1.0, dA, 2, M, dB, 2, N, 0.5, dC, 2, M) == 0
    out = from_dev(dC, "f16")
    assert blas.device_error() == 0
    assert _canary_ok(out, "f16", 0x5A5A), "wrote past the end of C"
    got = as_float(out[:-CANARY], "f16")
    ref = as_float(want, "f16")
    assert np.all(np.isfinite(got))
    err = normwise(got, ref)
    assert err <= 1e-2, err
    # both sides round once from fp32 accumulations: nearly every element
    # lands on the same fp16 value
    assert np.mean(out[:-CANARY] != want) < 0.05


def _batched_inputs():
    from zlift_b200 import inputs
    BATCH, M = 256, 512
    A = inputs.make("bf16", "normal", 201, BATCH * M * M)
    B = inputs.make("bf16", "normal", 202, BATCH * M * M)
    return BATCH, M, A, B


def test_strided_batched_bf16_256x512_full(handle, oracle_lib):
    """cublasGemmStridedBatchedEx bf16 256 x 512^3 NN, alpha 1/sqrt(512):
    every batch vs the oracle."""
    from zlift_b200 import blas
    BATCH, M, A, B = _batched_inputs()
    S = M * M
    alpha = 1.0 / math.sqrt(512)
    want = np.zeros(BATCH * S, np.uint16)
    assert oracle_lib.gemm_strided_batched_ex(0, 0, M, M, M, alpha, A, 14, M, S, B, 14, M, S,
                                              0.0, want, 14, M, S, BATCH) == 0
    dA, dB = to_dev(A, "bf16"), to_dev(B, "bf16")
    dC = to_dev(np.full(BATCH * S, 0x7FC1, np.uint16), "bf16", pad=CANARY, fill=0x5A5A)
    assert handle.gemm_strided_batched_ex(0, 0, M, M, M, alpha, dA, 14, M, S, dB, 14, M, S,
                                          0.0, dC, 14, M, S, BATCH) == 0
    out = from_dev(dC, "bf16")
    assert blas.device_error() == 0
    assert _canary_ok(out, "bf16", 0x5A5A), "wrote past the end of C"
    got = as_float(out[:-CANARY], "bf16").reshape(BATCH, S)
    ref = as_float(want, "bf16").reshape(BATCH, S)
    errs = [normwise(got[b], ref[b]) for b in range(BATCH)]
    assert max(errs) <= 1e-2, (int(np.argmax(errs)), max(errs))


def test_strided_batched_split_equals_one_shot(handle):
    """The batch split of the partition layer (two ranges on one GPU) gives
    the one-shot call's bits: same kernel, same tiles per matrix."""
    import torch
    from zlift_b200 import blas, partition
    BATCH, M, A, B = _batched_inputs()
    S = M * M
    alpha = 1.0 / math.sqrt(512)
    dA, dB = to_dev(A, "bf16"), to_dev(B, "bf16")
    one = torch.zeros(BATCH * S, dtype=torch.bfloat16, device="cuda")
    assert handle.gemm_strided_batched_ex(0, 0, M, M, M, alpha, dA, 14, M, S, dB, 14, M, S,
                                          0.0, one, 14, M, S, BATCH) == 0
    split = torch.zeros_like(one)
    for r in range(2):
        b0, b1 = partition.shard_range(BATCH, 2, r)
        assert partition.gemm_strided_batched_range(handle, b0, b1, 0, 0, M, M, M, alpha, dA,
                                                    14, M, S, dB, 14, M, S, 0.0, split, 14, M,
                                                    S, 68) == 0
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    assert torch.equal(one.view(torch.int16), split.view(torch.int16))


def test_gemm_ex_int8_2048x14336x4096_tn_bit_exact(handle, oracle_lib):
    """int8 x int8 -> int32 at 2048 x 14336 x 4096, TN: all of C bit-exact."""
    from zlift_b200 import blas, inputs
    M, K, N = 2048, 4096, 14336
    A = inputs.make("i8", "int8", 301, K * M)      # op T: stored K x M, lda = K
    B = inputs.make("i8", "int8", 302, K * N)      # op N: K x N, ldb = K
    want = np.zeros(M * N, np.int32)
    assert oracle_lib.gemm_ex(1, 0, M, N, K, 1, A, 3, K, B, 3, K, 0, want, 10, M, 72) == 0
    dA, dB = to_dev(A, "i8"), to_dev(B, "i8")
    dC = to_dev(np.full(M * N, -7, np.int32), "i32", pad=CANARY, fill=12345)
    assert handle.gemm_ex(1, 0, M, N, K, 1, dA, 3, K, dB, 3, K, 0, dC, 10, M,
                          compute=blas.COMPUTE_32I) == 0
    out = from_dev(dC, "i32")
    assert blas.device_error() == 0
    assert _canary_ok(out, "i32", 12345), "wrote past the end of C"
    np.testing.assert_array_equal(out[:-CANARY], want)


@pytest.mark.parametrize("ta,tb,m,n,k,alpha,beta", [
    (0, 1, 384, 256, 320, 1.0, 0.5),
    (1, 0, 200, 136, 96, -2.0, 0.0),
])
def test_hgemm(handle, oracle_lib, ta, tb, m, n, k, alpha, beta):
    """cublasHgemm (fp16 scalars, fp16 data) vs the oracle's fp16 GemmEx."""
    from zlift_b200 import blas, inputs
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    A = inputs.make("f16", "normal", 11, ar * ac, 0.125)
    B = inputs.make("f16", "normal", 12, br * bc, 0.125)
    C0 = inputs.make("f16", "normal", 13, m * n)
    want = C0.copy()
    assert oracle_lib.gemm_ex(ta, tb, m, n, k, alpha, A, 2, ar, B, 2, br, beta, want, 2, m) == 0
    a_bits = int(np.array([alpha], np.float16).view(np.uint16)[0])
    b_bits = int(np.array([beta], np.float16).view(np.uint16)[0])
    dA, dB, dC = to_dev(A, "f16"), to_dev(B, "f16"), to_dev(C0, "f16", pad=CANARY, fill=0x5A5A)
    assert handle.hgemm(ta, tb, m, n, k, a_bits, dA, ar, dB, br, b_bits, dC, m) == 0
    out = from_dev(dC, "f16")
    assert blas.device_error() == 0
    assert _canary_ok(out, "f16", 0x5A5A)
    assert normwise(as_float(out[:-CANARY], "f16"), as_float(want, "f16")) <= 1e-2


@pytest.mark.parametrize("kind,ckind", [("f16", "f16"), ("bf16", "bf16"), ("bf16", "f32"),
                                        ("f16", "f32")])
def test_sgemm_ex(handle, oracle_lib, kind, ckind):
    """cublasSgemmEx: 16-bit A/B, fp32 compute and scalars, 16-bit or fp32 C."""
    import ctypes
    from zlift_b200 import blas, inputs
    from tests.helpers import CUDA_T
    m, n, k = 300, 200, 272
    A = inputs.make(kind, "normal", 21, m * k, 0.25)
    B = inputs.make(kind, "normal", 22, k * n, 0.25)
    C0 = inputs.make(ckind, "normal", 23, m * n)
    want = C0.copy()
    assert oracle_lib.gemm_ex(0, 0, m, n, k, 0.75, A, CUDA_T[kind], m, B, CUDA_T[kind], k, 0.25,
                              want, CUDA_T[ckind], m) == 0
    dA, dB = to_dev(A, kind), to_dev(B, kind)
    fill = 0x5A5A if ckind != "f32" else 0
    dC = to_dev(C0, ckind, pad=CANARY, fill=fill)
    al, be = ctypes.c_float(0.75), ctypes.c_float(0.25)
    st = handle.lib.cublasSgemmEx(handle.h, 0, 0, m, n, k, ctypes.byref(al), dA.data_ptr(),
                                  CUDA_T[kind], m, dB.data_ptr(), CUDA_T[kind], k,
                                  ctypes.byref(be), dC.data_ptr(), CUDA_T[ckind], m)
    assert st == 0
    out = from_dev(dC, ckind)
    assert blas.device_error() == 0
    if ckind != "f32":
        assert _canary_ok(out, ckind, fill)
    got = as_float(out[:-CANARY], ckind)
    assert normwise(got, as_float(want, ckind)) <= 1e-2


def test_sgemm_strided_batched(handle, oracle_lib):
    """cublasSgemmStridedBatched (fp32, 3-product tf32) vs the oracle,
    normwise <= 1e-5 per batch."""
    from zlift_b200 import blas, inputs
    batch, m, n, k = 6, 160, 144, 200
    sA, sB, sC = m * k + 32, k * n + 16, m * n + 8          # padded batch strides
    A = inputs.make("f32", "uniform", 31, batch * sA)
    B = inputs.make("f32", "uniform", 32, batch * sB)
    C0 = inputs.make("f32", "uniform", 33, batch * sC)
    want = C0.copy()
    assert oracle_lib.gemm_strided_batched_ex(0, 1, m, n, k, 1.5, A, 0, m, sA, B, 0, n, sB,
                                              -0.5, want, 0, m, sC, batch) == 0
    dA, dB = to_dev(A, "f32"), to_dev(B, "f32")
    dC = to_dev(C0, "f32", pad=CANARY)
    dC[-CANARY:] = 12345.0
    assert handle.sgemm_strided_batched(0, 1, m, n, k, 1.5, dA, m, sA, dB, n, sB, -0.5, dC, m,
                                        sC, batch) == 0
    out = from_dev(dC, "f32")
    assert blas.device_error() == 0
    assert np.all(out[-CANARY:] == np.float32(12345.0))
    got = out[:-CANARY].astype(np.float64)
    ref = want.astype(np.float64)
    for b in range(batch):
        g = got[b * sC: b * sC + m * n]
        r = ref[b * sC: b * sC + m * n]
        assert normwise(g, r) <= 1e-5, b
        # the padding between matrices is left alone
        assert np.array_equal(got[b * sC + m * n:(b + 1) * sC], ref[b * sC + m * n:(b + 1) * sC])


def test_nsplit_overlap_one_rank_equals_one_shot(handle):
    """The overlapped N-split on one rank (no communicator): four sub-block
    GEMMs into their columns of C give the one-shot int8 product's bits."""
    import torch
    from zlift_b200 import blas, inputs, partition
    M, K, N = 512, 1024, 2048
    A = to_dev(inputs.make("i8", "int8", 401, K * M), "i8")
    Bh = inputs.make("i8", "int8", 402, K * N)
    B = to_dev(Bh, "i8")
    one = torch.zeros(N * M, dtype=torch.int32, device="cuda")
    assert handle.gemm_ex(1, 0, M, N, K, 1, A, 3, K, B, 3, K, 0, one, 10, M,
                          compute=blas.COMPUTE_32I) == 0
    SB = 4
    cols = [partition.nsplit_cols(N, 1, 0, SB, s) for s in range(SB)]
    Bcols = torch.cat([B[b * K:e * K] for b, e in cols])
    got = torch.full((N * M,), -1, dtype=torch.int32, device="cuda")
    assert partition.gemm_ex_nsplit_overlap(handle, None, 1, 0, SB, 1, 0, M, N, K, 1, A, 3, K,
                                            Bcols, 3, K, 0, got, 10, 72) == 0
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    assert torch.equal(one, got)


@pytest.mark.parametrize("ta,tb,m,n,k,alpha,beta", [
    (0, 0, 256, 192, 320, 1.0, 0.0),
    (1, 1, 100, 70, 131, -0.5, 2.0),
    (0, 1, 65, 257, 64, 2.0, 1.0),
])
def test_dgemm(handle, oracle_lib, ta, tb, m, n, k, alpha, beta):
    """cublasDgemm_v2 (zblas/zblas.c:131-144) vs the oracle's fp64 GEMM,
    normwise <= 1e-12 (both sum fp64 products, in different orders)."""
    import torch
    from zlift_b200 import blas, inputs
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    A = inputs.uniform(51, ar * ac)
    B = inputs.uniform(52, br * bc)
    C0 = inputs.uniform(53, m * n)
    want = C0.copy()
    oracle_lib.dgemm(ta, tb, m, n, k, alpha, A, ar, B, br, beta, want, m)
    dA = torch.from_numpy(A).cuda()
    dB = torch.from_numpy(B).cuda()
    dC = torch.from_numpy(np.concatenate([C0, np.full(CANARY, 7.0)])).cuda()
    assert handle.dgemm(ta, tb, m, n, k, alpha, dA, ar, dB, br, beta, dC, m) == 0
    out = dC.cpu().numpy()
    assert blas.device_error() == 0
    assert np.all(out[-CANARY:] == 7.0)
    assert normwise(out[:-CANARY], want) <= 1e-12


def test_fp16_output_edges(handle, oracle_lib):
    """fp16 outputs in the subnormal, overflow and NaN ranges, against the
    oracle's converter, which restates the reference's (zblas/zblas.c:
    260-277: round to nearest even for normals, truncation for subnormals,
    overflow to inf -- and NaN to inf too, since a NaN's exponent takes the
    overflow branch).  Deviations, stated here and bounded: the kernels
    round subnormals to nearest even, so a subnormal output may differ from
    the reference by one subnormal ulp (2^-24) and by no more; a NaN output
    stays NaN (IEEE, as NVIDIA's cuBLAS), where the reference writes inf.
    Overflows give the same infinities."""
    from zlift_b200 import blas, inputs
    m = n = 128
    k = 64
    A = inputs.make("f16", "uniform", 61, m * k)
    B = inputs.make("f16", "uniform", 62, k * n)
    Bf = inputs.bits_to_float(B, "f16").copy()
    Bf[5 * k + 3] = np.nan                         # column 5 of op(B) has a NaN
    B = Bf.astype(np.float16).view(np.uint16)
    for alpha, what in ((2.0 ** -18, "subnormal"), (2.0 ** 14, "overflow")):
        C0 = np.zeros(m * n, np.uint16)
        want = C0.copy()
        assert oracle_lib.gemm_ex(0, 0, m, n, k, alpha, A, 2, m, B, 2, k, 0.0, want, 2, m) == 0
        dA, dB = to_dev(A, "f16"), to_dev(B, "f16")
        dC = to_dev(C0, "f16")
        assert handle.gemm_ex(0, 0, m, n, k, alpha, dA, 2, m, dB, 2, k, 0.0, dC, 2, m) == 0
        got = from_dev(dC, "f16")
        assert blas.device_error() == 0
        g = got.view(np.float16).astype(np.float64)
        w = want.view(np.float16).astype(np.float64)
        col5 = np.zeros((n, m), bool)
        col5[5] = True
        col5 = col5.reshape(-1)
        assert np.isnan(g[col5]).all()                     # NaN stays NaN here ...
        assert np.isinf(w[col5]).all()                     # ... the reference writes inf
        assert not np.isnan(g[~col5]).any() and not np.isnan(w[~col5]).any()
        fin = ~col5
        inf_w = np.isinf(w) & fin
        np.testing.assert_array_equal(g[inf_w], w[inf_w])  # same infinities
        rest = fin & ~inf_w
        sub = rest & (np.abs(w) < 2.0 ** -14)
        if what == "subnormal":
            assert sub.sum() > m * n // 2                  # most outputs are subnormal
            assert np.max(np.abs(g[sub] - w[sub])) <= 2.0 ** -24
        else:
            assert inf_w.sum() > 0                         # some outputs overflowed
        nrm = rest & ~sub
        if nrm.any():
            # normal outputs: both round the same fp32 sum to nearest even,
            # up to the fp32 summation order
            assert normwise(g[nrm], w[nrm]) <= 1e-2
