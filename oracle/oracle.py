"""TEST INFRASTRUCTURE -- ctypes access to the oracle (the CPU checker).

Two libraries, both built by oracle/Makefile and neither ever loaded by the
product library:
  liboracle.so          the C restatement (zlift_oracle.c);
  _ref/libzblas_ref.so  the reference's own zblas/zblas.c CPU path,
                        compiled from its sources (only where the reference
                        tree was present at build time).
Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg import
this module.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_SO = os.path.join(HERE, "liboracle.so")
REF_SO = os.path.join(HERE, "_ref", "libzblas_ref.so")

R_32F, R_16F, R_8I, R_32I, R_16BF = 0, 2, 3, 10, 14
COMPUTE_32F, COMPUTE_32I = 68, 72

_vp, _int, _ll, _f, _d = (ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float,
                          ctypes.c_double)


def build(ref: bool = True) -> None:
    """Runs the Makefile: `make ref` builds the restatement and, where the
    reference sources are found (the recipe's REF), the reference's own CPU
    path; `make` only the restatement."""
    target = ["ref"] if ref else []
    subprocess.run(["make", "-s", "-C", HERE] + target, check=True,
                   stdout=subprocess.DEVNULL)


class AttnDesc(ctypes.Structure):
    _fields_ = [("q", _vp), ("k", _vp), ("v", _vp), ("o", _vp), ("lse", _vp),
                ("qb", _ll), ("qh", _ll), ("qr", _ll), ("kb", _ll), ("kh", _ll), ("kr", _ll),
                ("vb", _ll), ("vh", _ll), ("vr", _ll), ("ob", _ll), ("oh", _ll), ("orr", _ll),
                ("batch", _int), ("heads", _int), ("kv_ratio", _int), ("sq", _int),
                ("sk", _int), ("d", _int), ("scale", _f), ("causal", _int), ("diag", _int),
                ("elem", _int), ("bias", _vp), ("bb", _ll), ("bh", _ll), ("br", _ll)]


_oracle = None
_ref = None


def oracle() -> ctypes.CDLL:
    global _oracle
    if _oracle is None:
        if not os.path.exists(ORACLE_SO):
            build()
        lib = ctypes.CDLL(ORACLE_SO)
        lib.zo_gemm_ex.restype = _int
        lib.zo_gemm_ex.argtypes = [_int, _int, _int, _int, _int, _vp, _vp, _int, _int, _vp,
                                   _int, _int, _vp, _vp, _int, _int, _int]
        lib.zo_gemm_strided_batched_ex.restype = _int
        lib.zo_gemm_strided_batched_ex.argtypes = [_int, _int, _int, _int, _int, _vp, _vp,
                                                   _int, _int, _ll, _vp, _int, _int, _ll, _vp,
                                                   _vp, _int, _int, _ll, _int, _int]
        lib.zo_gemm_entries.restype = None
        lib.zo_gemm_entries.argtypes = [_int, _int, _int, _d, _vp, _int, _int, _vp, _int,
                                        _int, _d, _vp, _int, _int, _vp, _vp, _ll, _vp]
        lib.zo_dgemm.restype = None
        lib.zo_gemm_i8_s8.restype = _int
        lib.zo_gemm_i8_s8.argtypes = [_int, _int, _int, _int, _int, ctypes.c_float, _vp, _int,
                                      _vp, _int, ctypes.c_float, _vp, _int]
        lib.zo_dgemm.argtypes = [_int, _int, _int, _int, _int, _d, _vp, _int, _vp, _int, _d,
                                 _vp, _int]
        lib.zo_lt_epilogue.restype = None
        lib.zo_lt_epilogue.argtypes = [_vp, _int, _int, _int, _int, _ll, _int, _vp, _int]
        lib.zo_attention.restype = _int
        lib.zo_attention.argtypes = [ctypes.POINTER(AttnDesc)]
        lib.zo_attention_rows.restype = _int
        lib.zo_attention_rows.argtypes = [ctypes.POINTER(AttnDesc), _vp, _vp, _vp, _ll, _vp,
                                          _vp]
        assert lib.zo_attn_desc_size() == ctypes.sizeof(AttnDesc)
        for n in ("zo_half_to_float_n", "zo_bf16_to_float_n"):
            getattr(lib, n).argtypes = [_vp, _vp, _ll]
        for n in ("zo_float_to_half_n", "zo_float_to_bf16_n"):
            getattr(lib, n).argtypes = [_vp, _vp, _ll]
        _oracle = lib
    return _oracle


def ref_available() -> bool:
    return os.path.exists(REF_SO)


def reference() -> ctypes.CDLL:
    """The reference's zblas.c CPU path (cuBLAS C ABI on host memory)."""
    global _ref
    if _ref is None:
        lib = ctypes.CDLL(REF_SO, mode=os.RTLD_LOCAL | os.RTLD_NOW)
        lib.cublasCreate_v2.argtypes = [ctypes.POINTER(_vp)]
        lib.cublasSgemm_v2.argtypes = [_vp, _int, _int, _int, _int, _int, _vp, _vp, _int,
                                       _vp, _int, _vp, _vp, _int]
        lib.cublasGemmEx.argtypes = [_vp, _int, _int, _int, _int, _int, _vp, _vp, _int, _int,
                                     _vp, _int, _int, _vp, _vp, _int, _int, _int, _int]
        lib.cublasGemmStridedBatchedEx.argtypes = [_vp, _int, _int, _int, _int, _int, _vp,
                                                   _vp, _int, _int, _ll, _vp, _int, _int,
                                                   _ll, _vp, _vp, _int, _int, _ll, _int,
                                                   _int, _int]
        _ref = lib
    return _ref


def _p(a: np.ndarray) -> int:
    return a.ctypes.data


def _scalar(v, integer):
    return np.array([v], dtype=np.int32 if integer else np.float32)


def gemm_ex(transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype,
            ldc, compute=COMPUTE_32F) -> int:
    """Oracle restatement of cublasGemmEx on host arrays (C updated in place)."""
    integer = compute in (COMPUTE_32I, R_32I)
    al, be = _scalar(alpha, integer), _scalar(beta, integer)
    return oracle().zo_gemm_ex(transa, transb, m, n, k, _p(al), _p(A), Atype, lda, _p(B),
                               Btype, ldb, _p(be), _p(C), Ctype, ldc, compute)


def gemm_strided_batched_ex(transa, transb, m, n, k, alpha, A, Atype, lda, sA, B, Btype, ldb,
                            sB, beta, C, Ctype, ldc, sC, batch, compute=COMPUTE_32F) -> int:
    integer = compute in (COMPUTE_32I, R_32I)
    al, be = _scalar(alpha, integer), _scalar(beta, integer)
    return oracle().zo_gemm_strided_batched_ex(transa, transb, m, n, k, _p(al), _p(A), Atype,
                                               lda, sA, _p(B), Btype, ldb, sB, _p(be), _p(C),
                                               Ctype, ldc, sC, batch, compute)


def gemm_i8_s8(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    """int8 C = sat_s8(rne(alpha * op(A) op(B) + beta * C)), float alpha/beta (in place)."""
    assert A.dtype == np.int8 and B.dtype == np.int8 and C.dtype == np.int8
    return oracle().zo_gemm_i8_s8(transa, transb, m, n, k, float(alpha), _p(A), lda, _p(B), ldb,
                                  float(beta), _p(C), ldc)


def dgemm(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> None:
    """Oracle restatement of cublasDgemm_v2 on host float64 arrays (C in place)."""
    oracle().zo_dgemm(transa, transb, m, n, k, float(alpha), _p(A), lda, _p(B), ldb,
                      float(beta), _p(C), ldc)


def lt_epilogue(D, Dtype, m, n, ldd, strideD, batch, bias, flags) -> None:
    """The reference's cublasLtMatmul epilogue on host D (in place)."""
    oracle().zo_lt_epilogue(_p(D), Dtype, m, n, ldd, strideD, batch,
                            _p(bias) if bias is not None else None, flags)


def gemm_entries(transa, transb, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C0, Ctype, ldc,
                 rows, cols) -> np.ndarray:
    """fp64 values of alpha*op(A)op(B) + beta*C0 at (rows[t], cols[t])."""
    rows = np.ascontiguousarray(rows, dtype=np.int64)
    cols = np.ascontiguousarray(cols, dtype=np.int64)
    out = np.zeros(len(rows), dtype=np.float64)
    oracle().zo_gemm_entries(transa, transb, k, float(alpha), _p(A), Atype, lda, _p(B), Btype,
                             ldb, float(beta), _p(C0) if C0 is not None else None, Ctype, ldc,
                             _p(rows), _p(cols), len(rows), _p(out))
    return out


def ref_gemm_ex(transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb, beta, C, Ctype,
                ldc, compute=COMPUTE_32F) -> int:
    """The reference's own cublasGemmEx (CPU path) on host arrays."""
    lib = reference()
    h = _vp()
    assert lib.cublasCreate_v2(ctypes.byref(h)) == 0
    integer = compute in (COMPUTE_32I, R_32I)
    al, be = _scalar(alpha, integer), _scalar(beta, integer)
    rc = lib.cublasGemmEx(h, transa, transb, m, n, k, _p(al), _p(A), Atype, lda, _p(B), Btype,
                          ldb, _p(be), _p(C), Ctype, ldc, compute, 0)
    lib.cublasDestroy_v2(h)
    return rc


def ref_sgemm(transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
    lib = reference()
    h = _vp()
    assert lib.cublasCreate_v2(ctypes.byref(h)) == 0
    al, be = _scalar(alpha, False), _scalar(beta, False)
    rc = lib.cublasSgemm_v2(h, transa, transb, m, n, k, _p(al), _p(A), lda, _p(B), ldb, _p(be),
                            _p(C), ldc)
    lib.cublasDestroy_v2(h)
    return rc


def ref_gemm_strided_batched_ex(transa, transb, m, n, k, alpha, A, Atype, lda, sA, B, Btype,
                                ldb, sB, beta, C, Ctype, ldc, sC, batch,
                                compute=COMPUTE_32F) -> int:
    lib = reference()
    h = _vp()
    assert lib.cublasCreate_v2(ctypes.byref(h)) == 0
    al, be = _scalar(alpha, False), _scalar(beta, False)
    rc = lib.cublasGemmStridedBatchedEx(h, transa, transb, m, n, k, _p(al), _p(A), Atype, lda,
                                        sA, _p(B), Btype, ldb, sB, _p(be), _p(C), Ctype, ldc,
                                        sC, batch, compute, 0)
    lib.cublasDestroy_v2(h)
    return rc


def attention(q, k, v, causal, scale, elem, kv_ratio=1, diag=None, want_lse=True, bias=None):
    """Oracle attention on host arrays laid out [B, S, H, D] (16-bit values
    as uint16 bit patterns, fp32 as float32).  `bias`, if given, is an array
    [B, H, Sq, Sk] of the input type added to the scaled scores.  Returns
    (O, LSE[B, H, Sq])."""
    B, Sq, H, D = q.shape
    Sk = k.shape[1]
    o = np.zeros_like(q)
    lse = np.zeros((B, H, Sq), dtype=np.float32)
    d = _desc(q, k, v, o, lse if want_lse else None, causal, scale, elem, kv_ratio, diag, bias)
    rc = oracle().zo_attention(ctypes.byref(d))
    assert rc == 0
    return o, lse


def attention_rows(q, k, v, causal, scale, elem, bs, hs, is_, kv_ratio=1, diag=None, bias=None):
    """fp64 O rows and LSE values for selected (b, h, i) query rows."""
    D = q.shape[3]
    d = _desc(q, k, v, None, None, causal, scale, elem, kv_ratio, diag, bias)
    bs = np.ascontiguousarray(bs, dtype=np.int32)
    hs = np.ascontiguousarray(hs, dtype=np.int32)
    is_ = np.ascontiguousarray(is_, dtype=np.int32)
    o = np.zeros((len(bs), D), dtype=np.float64)
    l = np.zeros(len(bs), dtype=np.float64)
    rc = oracle().zo_attention_rows(ctypes.byref(d), _p(bs), _p(hs), _p(is_), len(bs), _p(o),
                                    _p(l))
    assert rc == 0
    return o, l


def _desc(q, k, v, o, lse, causal, scale, elem, kv_ratio, diag, bias=None):
    B, Sq, H, D = q.shape
    Sk = k.shape[1]
    d = AttnDesc()
    d.q, d.k, d.v = _p(q), _p(k), _p(v)
    d.o = _p(o) if o is not None else None
    d.lse = _p(lse) if lse is not None else None
    es = q.itemsize
    d.qb, d.qr, d.qh = (s // es for s in q.strides[:3])
    d.kb, d.kr, d.kh = (s // es for s in k.strides[:3])
    d.vb, d.vr, d.vh = (s // es for s in v.strides[:3])
    if o is not None:
        d.ob, d.orr, d.oh = (s // es for s in o.strides[:3])
    d.batch, d.heads, d.kv_ratio, d.sq, d.sk, d.d = B, H, kv_ratio, Sq, Sk, D
    d.scale = scale
    d.causal = 1 if causal else 0
    d.diag = (Sk - Sq) if diag is None else diag
    d.elem = elem
    if bias is not None:
        assert bias.shape == (B, H, Sq, Sk) and bias.dtype == q.dtype
        d.bias = _p(bias)
        d.bb, d.bh, d.br = (s // bias.itemsize for s in bias.strides[:3])
    return d


# converters (zblas/zblas.c:241-277, :306-317), array forms
def half_to_float(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, dtype=np.float32)
    oracle().zo_half_to_float_n(_p(x), _p(y), x.size)
    return y


def float_to_half(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    oracle().zo_float_to_half_n(_p(x), _p(y), x.size)
    return y


def bf16_to_float(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.uint16)
    y = np.empty(x.shape, dtype=np.float32)
    oracle().zo_bf16_to_float_n(_p(x), _p(y), x.size)
    return y


def float_to_bf16(x: np.ndarray) -> np.ndarray:
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.empty(x.shape, dtype=np.uint16)
    oracle().zo_float_to_bf16_n(_p(x), _p(y), x.size)
    return y
