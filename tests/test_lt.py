"""cuBLASLt subset (include/zlift_cublaslt.h).

CPU: descriptor / layout / preference / heuristic calls and the
NOT_SUPPORTED stubs, all answered on the host.
GPU: cublasLtMatmul with every epilogue (none, bias, ReLU, bias+ReLU, GELU,
bias+GELU) against the oracle's restatement of the reference -- its GEMM
(gemm_ex_host) followed by its host epilogue (zblas/zblas.c:692-710) --
within the fp16/bf16 GEMM tolerance (normwise <= 1e-2; the reference
rounds D to 16 bits before the epilogue, this library applies the epilogue
in fp32 and rounds once).
"""
import ctypes
import re
import os

import numpy as np
import pytest

from tests.helpers import CUDA_T, as_float, from_dev, normwise, to_dev

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
vp, ci, cs, cll, cull = (ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t, ctypes.c_longlong,
                         ctypes.c_ulonglong)


def _lt(lib):
    lib.cublasLtMatmulDescCreate.argtypes = [ctypes.POINTER(vp), ci, ci]
    lib.cublasLtMatmulDescSetAttribute.argtypes = [vp, ci, vp, cs]
    lib.cublasLtMatmulDescGetAttribute.argtypes = [vp, ci, vp, cs, ctypes.POINTER(cs)]
    lib.cublasLtMatrixLayoutCreate.argtypes = [ctypes.POINTER(vp), ci, cull, cull, cll]
    lib.cublasLtMatrixLayoutSetAttribute.argtypes = [vp, ci, vp, cs]
    lib.cublasLtMatmulPreferenceCreate.argtypes = [ctypes.POINTER(vp)]
    lib.cublasLtMatmulAlgoGetHeuristic.argtypes = [vp, vp, vp, vp, vp, vp, vp, ci, vp,
                                                   ctypes.POINTER(ci)]
    lib.cublasLtMatmul.argtypes = [vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, cs, vp]
    lib.cublasLtCreate.argtypes = [ctypes.POINTER(vp)]
    lib.cublasLtDestroy.argtypes = [vp]
    lib.cublasLtMatmulDescDestroy.argtypes = [vp]
    lib.cublasLtMatrixLayoutDestroy.argtypes = [vp]
    return lib


def _set(lib, desc, attr, value, ctype=ci):
    v = ctype(value)
    return lib.cublasLtMatmulDescSetAttribute(desc, attr, ctypes.byref(v), ctypes.sizeof(v))


def _layout(lib, t, rows, cols, ld, batch=1, stride=0):
    l = vp()
    assert lib.cublasLtMatrixLayoutCreate(ctypes.byref(l), t, rows, cols, ld) == 0
    if batch > 1:
        b, s = ci(batch), cll(stride)
        assert lib.cublasLtMatrixLayoutSetAttribute(l, 5, ctypes.byref(b), 4) == 0
        assert lib.cublasLtMatrixLayoutSetAttribute(l, 6, ctypes.byref(s), 8) == 0
    return l


def test_lt_descriptors_on_host(built_lib):
    lib = _lt(built_lib)
    assert lib.cublasLtGetVersion() == 130100
    d = vp()
    assert lib.cublasLtMatmulDescCreate(ctypes.byref(d), 68, 0) == 0
    assert _set(lib, d, 3, 1) == 0 and _set(lib, d, 7, 36) == 0
    out, w = ci(), cs()
    assert lib.cublasLtMatmulDescGetAttribute(d, 3, ctypes.byref(out), 4, ctypes.byref(w)) == 0
    assert out.value == 1 and w.value == 4
    assert lib.cublasLtMatmulDescGetAttribute(d, 7, ctypes.byref(out), 4, None) == 0
    assert out.value == 36
    assert lib.cublasLtMatmulDescGetAttribute(d, 7, ctypes.byref(out), 2, None) == 7
    assert lib.cublasLtMatmulDescSetAttribute(d, 7, None, 4) == 7
    p = vp()
    assert lib.cublasLtMatmulPreferenceCreate(ctypes.byref(p)) == 0
    res = (ctypes.c_ubyte * 96)()
    n = ci()
    assert lib.cublasLtMatmulAlgoGetHeuristic(None, d, None, None, None, None, p, 1, res,
                                              ctypes.byref(n)) == 0
    assert n.value == 1
    lib.cublasLtMatmulPreferenceDestroy(p)
    assert lib.cublasLtMatmulDescDestroy(d) == 0


def test_lt_rejects_on_host(built_lib):
    lib = _lt(built_lib)
    h = vp()
    assert lib.cublasLtCreate(ctypes.byref(h)) == 0
    d = vp()
    lib.cublasLtMatmulDescCreate(ctypes.byref(d), 68, 0)
    la, lb, lc = _layout(lib, 2, 8, 8, 8), _layout(lib, 2, 8, 8, 8), _layout(lib, 2, 8, 8, 8)
    one = ctypes.c_float(1.0)
    call = lambda: lib.cublasLtMatmul(h, d, ctypes.byref(one), 16, la, 16, lb,
                                      ctypes.byref(one), 16, lc, 16, lc, None, None, 0, None)
    _set(lib, d, 7, 99)
    assert call() == 15                         # unknown epilogue
    _set(lib, d, 7, 4)
    assert call() == 7                          # bias epilogue without a bias pointer
    _set(lib, d, 7, 1)
    order = ci(1)                               # row-major layouts are not supported
    lib.cublasLtMatrixLayoutSetAttribute(la, 1, ctypes.byref(order), 4)
    assert call() == 15
    lb2 = _layout(lib, 2, 9, 8, 9)              # B rows disagree with k
    order.value = 0
    lib.cublasLtMatrixLayoutSetAttribute(la, 1, ctypes.byref(order), 4)
    assert lib.cublasLtMatmul(h, d, ctypes.byref(one), 16, la, 16, lb2, ctypes.byref(one), 16,
                              lc, 16, lc, None, None, 0, None) == 7
    assert lib.cublasLtMatmul(None, d, ctypes.byref(one), 16, la, 16, lb, ctypes.byref(one), 16,
                              lc, 16, lc, None, None, 0, None) == 1
    for l in (la, lb, lc, lb2):
        lib.cublasLtMatrixLayoutDestroy(l)
    lib.cublasLtMatmulDescDestroy(d)
    lib.cublasLtDestroy(h)


def _stub_names():
    src = open(os.path.join(ROOT, "include", "zlift_cublaslt.h")).read()
    block = src[src.index("#define ZLIFT_UNSUPPORTED_LIST"):src.index("#define ZLIFT_DECLARE")]
    return re.findall(r"X\((cublas\w+)\)", block)


def test_unsupported_stubs_exported_and_answer_15(built_lib):
    names = _stub_names()
    assert len(names) == 36
    for n in names:
        fn = getattr(built_lib, n)
        fn.restype = ci
        fn.argtypes = []
        assert fn() == 15, n


GPU_CASES = [
    # (kind, ta, tb, m, n, k, epilogue, alpha, beta, c_is_d, batch)
    ("f16", 0, 1, 256, 320, 192, 1, 1.0, 0.5, True, 1),
    ("bf16", 1, 0, 200, 136, 96, 4, 1.0, 0.0, True, 1),
    ("f16", 0, 0, 128, 256, 64, 2, 0.5, 0.0, True, 1),
    ("bf16", 0, 1, 300, 260, 200, 6, 1.0, 1.0, False, 1),
    ("f16", 1, 1, 96, 80, 48, 32, 1.0, 0.0, True, 1),
    ("bf16", 0, 0, 512, 384, 256, 36, 0.25, 0.5, False, 1),
    ("bf16", 0, 0, 128, 128, 64, 36, 1.0, 0.0, True, 3),
    ("f32", 0, 1, 64, 96, 80, 6, 1.0, 0.0, True, 1),
]


@pytest.mark.gpu
@pytest.mark.parametrize("kind,ta,tb,m,n,k,epi,alpha,beta,c_is_d,batch", GPU_CASES)
def test_lt_matmul_epilogues(built_lib, oracle_lib, cuda, kind, ta, tb, m, n, k, epi, alpha,
                             beta, c_is_d, batch):
    import torch
    from zlift_b200 import inputs
    lib = _lt(built_lib)
    T = CUDA_T[kind]
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    sA, sB, sC = ar * ac, br * bc, m * n
    A = inputs.make(kind, "normal", 1, sA * batch, 0.25)
    B = inputs.make(kind, "normal", 2, sB * batch, 0.25)
    C0 = inputs.make(kind, "normal", 3, sC * batch)
    bias = inputs.make(kind, "normal", 4, m)
    # oracle: GEMM into D (= C), then the reference's epilogue on D
    want = C0.copy()
    rc = oracle_lib.gemm_strided_batched_ex(ta, tb, m, n, k, alpha, A, T, ar, sA, B, T, br, sB,
                                            beta, want, T, m, sC, batch)
    assert rc == 0
    flags = (1 if epi in (4, 6, 36) else 0) | (2 if epi in (2, 6) else 0) | \
            (4 if epi in (32, 36) else 0)
    oracle_lib.lt_epilogue(want, T, m, n, m, sC, batch, bias, flags)
    # GPU
    h = vp()
    assert lib.cublasLtCreate(ctypes.byref(h)) == 0
    d = vp()
    lib.cublasLtMatmulDescCreate(ctypes.byref(d), 68, 0)
    _set(lib, d, 3, ta)
    _set(lib, d, 4, tb)
    _set(lib, d, 7, epi)
    dA, dB, dBias = to_dev(A, kind), to_dev(B, kind), to_dev(bias, kind)
    _set(lib, d, 8, dBias.data_ptr(), vp)
    dC = to_dev(C0, kind)
    dD = dC if c_is_d else to_dev(np.zeros_like(C0), kind)
    la = _layout(lib, T, ar, ac, ar, batch, sA)
    lb = _layout(lib, T, br, bc, br, batch, sB)
    lc = _layout(lib, T, m, n, m, batch, sC)
    al, be = ctypes.c_float(alpha), ctypes.c_float(beta)
    s = torch.cuda.current_stream().cuda_stream
    st = lib.cublasLtMatmul(h, d, ctypes.byref(al), dA.data_ptr(), la, dB.data_ptr(), lb,
                            ctypes.byref(be), dC.data_ptr(), lc, dD.data_ptr(), lc, None, None,
                            0, s)
    assert st == 0
    torch.cuda.synchronize()
    got = as_float(from_dev(dD, kind), kind)
    ref = as_float(want, kind)
    assert normwise(got, ref) <= (1e-2 if kind != "f32" else 1e-5)
    if not c_is_d:
        np.testing.assert_array_equal(from_dev(dC, kind), C0)   # C is not written
    for l in (la, lb, lc):
        lib.cublasLtMatrixLayoutDestroy(l)
    lib.cublasLtMatmulDescDestroy(d)
    lib.cublasLtDestroy(h)


# ---------------------------------------------------------------------------
# int8 output (requantising epilogue): int8 A/B/C/D, compute 32I, scale 32F.
# D = sat_s8(rne(alpha * float(acc) + beta * float(C))), bit-exact.

def _requant_np(A, B, C0, ta, tb, m, n, k, alpha, beta):
    """numpy restatement: exact int64 product, one float32 multiply, the
    beta term added in float64 (exact for the power-of-two betas used here,
    so it equals the single rounding of fmaf), ties to even, saturation."""
    opA = (A.reshape(m, k, order="F") if ta == 0 else A.reshape(k, m, order="F").T).astype(np.int64)
    opB = (B.reshape(k, n, order="F") if tb == 0 else B.reshape(n, k, order="F").T).astype(np.int64)
    acc = (opA @ opB).astype(np.int32)
    x = np.float32(alpha) * acc.astype(np.float32)
    if beta != 0.0:
        c = C0.reshape(m, n, order="F").astype(np.float64)
        x = (np.float64(beta) * c + x.astype(np.float64)).astype(np.float32)
    out = np.clip(np.rint(x), -128, 127).astype(np.int8)
    return out.reshape(-1, order="F")


@pytest.mark.parametrize("ta,tb,alpha,beta", [(1, 0, 0.5, 0.0), (0, 1, 0.013, 0.5),
                                              (0, 0, 3.0, -0.25), (1, 1, 0.0071, 1.0)])
def test_oracle_requant_matches_numpy(oracle_lib, ta, tb, alpha, beta):
    """The oracle's int8-output GEMM: ties to even (alpha 0.5 makes every odd
    accumulator a tie), saturation (alpha 3), and the beta term."""
    from zlift_b200 import inputs
    m, n, k = 37, 29, 70
    A = inputs.make("i8", "int8", 91, m * k)
    B = inputs.make("i8", "int8", 92, k * n)
    C0 = inputs.make("i8", "int8", 93, m * n)
    got = C0.copy()
    assert oracle_lib.gemm_i8_s8(ta, tb, m, n, k, alpha, A, m if ta == 0 else k, B,
                                 k if tb == 0 else n, beta, got, m) == 0
    want = _requant_np(A, B, C0, ta, tb, m, n, k, alpha, beta)
    np.testing.assert_array_equal(got, want)
    if alpha == 3.0:
        assert (got == 127).any() and (got == -128).any()


I8_CASES = [
    # (ta, tb, m, n, k, alpha, beta, ldc_pad, c_is_d): staged TMA epilogue,
    # direct stores (ldc not a multiple of 16), the CUDA-core kernel (odd
    # lda), a K-split shape (few tiles, long K), MN-major operands
    (1, 0, 256, 384, 512, 0.01, 0.0, 0, True),
    (1, 0, 512, 256, 1024, 0.003, 0.5, 0, False),
    (1, 0, 200, 136, 256, 0.02, -0.25, 3, True),
    (1, 0, 96, 80, 61, 0.05, 1.0, 0, True),
    (1, 0, 128, 128, 8192, 0.0004, 0.5, 0, True),
    (0, 1, 256, 256, 384, 0.01, 0.0, 0, True),
    (0, 0, 256, 256, 256, 0.5, 0.0, 0, True),
]


@pytest.mark.gpu
@pytest.mark.parametrize("ta,tb,m,n,k,alpha,beta,pad,c_is_d", I8_CASES)
def test_lt_matmul_int8_out(built_lib, oracle_lib, cuda, ta, tb, m, n, k, alpha, beta, pad,
                            c_is_d):
    import torch
    from zlift_b200 import inputs
    lib = _lt(built_lib)
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    ldc = m + pad
    A = inputs.make("i8", "int8", 101, ar * ac)
    B = inputs.make("i8", "int8", 102, br * bc)
    C0 = inputs.make("i8", "int8", 103, ldc * n)
    want = C0.copy()
    assert oracle_lib.gemm_i8_s8(ta, tb, m, n, k, alpha, A, ar, B, br, beta, want, ldc) == 0
    h = vp()
    assert lib.cublasLtCreate(ctypes.byref(h)) == 0
    d = vp()
    assert lib.cublasLtMatmulDescCreate(ctypes.byref(d), 72, 0) == 0     # 32I compute, 32F scale
    _set(lib, d, 3, ta)
    _set(lib, d, 4, tb)
    dA, dB = to_dev(A, "i8"), to_dev(B, "i8")
    dC = to_dev(C0, "i8")
    dD = dC if c_is_d else to_dev(np.zeros_like(C0), "i8")
    la = _layout(lib, 3, ar, ac, ar)
    lb = _layout(lib, 3, br, bc, br)
    lc = _layout(lib, 3, m, n, ldc)
    al, be = ctypes.c_float(alpha), ctypes.c_float(beta)
    s = torch.cuda.current_stream().cuda_stream
    st = lib.cublasLtMatmul(h, d, ctypes.byref(al), dA.data_ptr(), la, dB.data_ptr(), lb,
                            ctypes.byref(be), dC.data_ptr(), lc, dD.data_ptr(), lc, None, None,
                            0, s)
    assert st == 0
    torch.cuda.synchronize()
    from zlift_b200 import blas
    assert blas.device_error() == 0
    got = from_dev(dD, "i8").reshape(n, ldc)
    np.testing.assert_array_equal(got[:, :m], want.reshape(n, ldc)[:, :m])
    if alpha >= 0.5:
        assert (got[:, :m] == 127).any() or (got[:, :m] == -128).any()
    if not c_is_d:
        np.testing.assert_array_equal(from_dev(dC, "i8"), C0)
    for l in (la, lb, lc):
        lib.cublasLtMatrixLayoutDestroy(l)
    lib.cublasLtMatmulDescDestroy(d)
    lib.cublasLtDestroy(h)


def test_lt_int8_out_rejections_on_host(built_lib):
    """int8 D needs scale type 32F, takes no bias/activation epilogue, and
    cublasGemmEx itself has no int8 output (NOT_SUPPORTED, as cuBLAS)."""
    lib = _lt(built_lib)
    h = vp()
    assert lib.cublasLtCreate(ctypes.byref(h)) == 0
    d = vp()
    assert lib.cublasLtMatmulDescCreate(ctypes.byref(d), 72, 10) == 0    # scale type 32I
    l = _layout(lib, 3, 16, 16, 16)
    one = ctypes.c_float(1.0)
    call = lambda: lib.cublasLtMatmul(h, d, ctypes.byref(one), 16, l, 16, l, ctypes.byref(one),
                                      16, l, 16, l, None, None, 0, None)
    assert call() == 15
    _set(lib, d, 1, 0)                         # scale type 32F
    _set(lib, d, 7, 2)                         # ReLU epilogue
    assert call() == 15
    hb = vp()
    built_lib.cublasCreate_v2.argtypes = [ctypes.POINTER(vp)]
    assert built_lib.cublasCreate_v2(ctypes.byref(hb)) == 0
    built_lib.cublasGemmEx.argtypes = [vp, ci, ci, ci, ci, ci, vp, vp, ci, ci, vp, ci, ci, vp,
                                       vp, ci, ci, ci, ci]
    assert built_lib.cublasGemmEx(hb, 1, 0, 16, 16, 16, ctypes.byref(one), 16, 3, 16, 16, 3, 16,
                                  ctypes.byref(one), 16, 3, 16, 72, 0) == 15
    built_lib.cublasDestroy_v2.argtypes = [vp]
    built_lib.cublasDestroy_v2(hb)
    lib.cublasLtMatrixLayoutDestroy(l)
    lib.cublasLtMatmulDescDestroy(d)
    lib.cublasLtDestroy(h)


@pytest.mark.gpu
@pytest.mark.parametrize("device_scalars", [False, True])
def test_lt_matmul_int8_out_batched(built_lib, oracle_lib, cuda, device_scalars):
    """int8 output over batched layouts (3 batches, padded batch strides), with
    alpha/beta read on the host or from device memory (pointer mode device),
    bit-exact per batch against the oracle."""
    import torch
    from zlift_b200 import inputs
    lib = _lt(built_lib)
    ta, tb, m, n, k, batch = 1, 0, 192, 160, 320, 3
    alpha, beta = 0.0123, 0.5
    sA, sB, sC = k * m + 64, k * n + 32, m * n + 16
    A = inputs.make("i8", "int8", 111, sA * batch)
    B = inputs.make("i8", "int8", 112, sB * batch)
    C0 = inputs.make("i8", "int8", 113, sC * batch)
    want = C0.copy()
    for b in range(batch):
        cb = want[b * sC:b * sC + m * n].copy()
        assert oracle_lib.gemm_i8_s8(ta, tb, m, n, k, alpha, A[b * sA:], k, B[b * sB:], k, beta,
                                     cb, m) == 0
        want[b * sC:b * sC + m * n] = cb
    h = vp()
    assert lib.cublasLtCreate(ctypes.byref(h)) == 0
    d = vp()
    assert lib.cublasLtMatmulDescCreate(ctypes.byref(d), 72, 0) == 0
    _set(lib, d, 3, ta)
    _set(lib, d, 4, tb)
    dA, dB, dC = to_dev(A, "i8"), to_dev(B, "i8"), to_dev(C0, "i8")
    la = _layout(lib, 3, k, m, k, batch, sA)
    lb = _layout(lib, 3, k, n, k, batch, sB)
    lc = _layout(lib, 3, m, n, m, batch, sC)
    s = torch.cuda.current_stream().cuda_stream
    if device_scalars:
        _set(lib, d, 2, 1)                                    # CUBLAS_POINTER_MODE_DEVICE
        scal = torch.tensor([alpha, beta], dtype=torch.float32, device="cuda")
        pa, pb = scal.data_ptr(), scal.data_ptr() + 4
    else:
        al, be = ctypes.c_float(alpha), ctypes.c_float(beta)
        pa, pb = ctypes.addressof(al), ctypes.addressof(be)
    st = lib.cublasLtMatmul(h, d, pa, dA.data_ptr(), la, dB.data_ptr(), lb, pb, dC.data_ptr(),
                            lc, dC.data_ptr(), lc, None, None, 0, s)
    assert st == 0
    torch.cuda.synchronize()
    from zlift_b200 import blas
    assert blas.device_error() == 0
    got = from_dev(dC, "i8")
    np.testing.assert_array_equal(got, want)      # the padding between batches is untouched too
    for l in (la, lb, lc):
        lib.cublasLtMatrixLayoutDestroy(l)
    lib.cublasLtMatmulDescDestroy(d)
    lib.cublasLtDestroy(h)
