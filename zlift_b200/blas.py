"""Python mirror of the cuBLAS-style C ABI in libcublas.so.13.

Names, argument order and meaning follow zLift's zblas/zblas.c (column-major
operands, leading dimensions and batch strides in elements, status codes
0/1/7/13/15).  Operands are device addresses (ints) or anything with a
``data_ptr()`` method (torch tensors); host scalars are Python numbers.
"""
from __future__ import annotations

import ctypes

from . import load

SUCCESS, NOT_INITIALIZED, INVALID_VALUE, EXECUTION_FAILED, NOT_SUPPORTED = 0, 1, 7, 13, 15
OP_N, OP_T, OP_C = 0, 1, 2
R_32F, R_16F, R_8I, R_32I, R_16BF = 0, 2, 3, 10, 14
COMPUTE_32F, COMPUTE_32I = 68, 72
POINTER_MODE_HOST, POINTER_MODE_DEVICE = 0, 1
DEFAULT_MATH, TF32_TENSOR_OP_MATH = 0, 3


class GemmError(RuntimeError):
    def __init__(self, status: int, what: str):
        name = load().cublasGetStatusName(status).decode()
        super().__init__(f"{what}: {name} ({status})")
        self.status = status


def _ptr(x) -> int:
    if x is None:
        return 0
    if isinstance(x, int):
        return x
    return int(x.data_ptr())


def _stream_ptr(stream) -> int:
    if stream is None:
        return 0
    if isinstance(stream, int):
        return stream
    return int(getattr(stream, "cuda_stream", 0))


class Handle:
    """A cuBLAS handle of this library (cublasCreate_v2 ... cublasDestroy_v2)."""

    def __init__(self, stream=None):
        self.lib = load()
        h = ctypes.c_void_p()
        st = self.lib.cublasCreate_v2(ctypes.byref(h))
        if st:
            raise GemmError(st, "cublasCreate_v2")
        self.h = h
        self._keep = []
        if stream is not None:
            self.set_stream(stream)

    def close(self):
        if self.h:
            self.lib.cublasDestroy_v2(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    # ---- handle state ----
    def set_stream(self, stream):
        st = self.lib.cublasSetStream_v2(self.h, _stream_ptr(stream))
        if st:
            raise GemmError(st, "cublasSetStream_v2")

    def set_pointer_mode(self, mode: int):
        return self.lib.cublasSetPointerMode_v2(self.h, mode)

    def set_math_mode(self, mode: int):
        return self.lib.cublasSetMathMode(self.h, mode)

    def set_workspace(self, ptr, nbytes: int):
        return self.lib.cublasSetWorkspace_v2(self.h, _ptr(ptr), nbytes)

    # ---- scalars ----
    def _scalar(self, v, integer: bool):
        """Host value -> pointer to a ctypes scalar; an int address or a
        tensor passes through as a device pointer (device pointer mode)."""
        if hasattr(v, "data_ptr"):
            return ctypes.c_void_p(_ptr(v))
        if integer:
            s = ctypes.c_int32(int(v))
        else:
            s = ctypes.c_float(float(v))
        self._keep.append(s)
        return ctypes.cast(ctypes.byref(s), ctypes.c_void_p)

    # ---- GEMM entry points (return the status, never raise) ----
    def sgemm(self, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
        self._keep.clear()
        return self.lib.cublasSgemm_v2(self.h, transa, transb, m, n, k,
                                       self._scalar(alpha, False), _ptr(A), lda, _ptr(B), ldb,
                                       self._scalar(beta, False), _ptr(C), ldc)

    def dgemm(self, transa, transb, m, n, k, alpha, A, lda, B, ldb, beta, C, ldc) -> int:
        al, be = ctypes.c_double(float(alpha)), ctypes.c_double(float(beta))
        return self.lib.cublasDgemm_v2(self.h, transa, transb, m, n, k, ctypes.byref(al),
                                       _ptr(A), lda, _ptr(B), ldb, ctypes.byref(be), _ptr(C),
                                       ldc)

    def gemm_ex(self, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb,
                beta, C, Ctype, ldc, compute=COMPUTE_32F, algo=0) -> int:
        self._keep.clear()
        integer = compute in (COMPUTE_32I, R_32I)
        return self.lib.cublasGemmEx(self.h, transa, transb, m, n, k,
                                     self._scalar(alpha, integer), _ptr(A), Atype, lda,
                                     _ptr(B), Btype, ldb, self._scalar(beta, integer),
                                     _ptr(C), Ctype, ldc, compute, algo)

    def gemm_strided_batched_ex(self, transa, transb, m, n, k, alpha, A, Atype, lda, sA,
                                B, Btype, ldb, sB, beta, C, Ctype, ldc, sC, batch,
                                compute=COMPUTE_32F, algo=0) -> int:
        self._keep.clear()
        integer = compute in (COMPUTE_32I, R_32I)
        return self.lib.cublasGemmStridedBatchedEx(
            self.h, transa, transb, m, n, k, self._scalar(alpha, integer), _ptr(A), Atype,
            lda, sA, _ptr(B), Btype, ldb, sB, self._scalar(beta, integer), _ptr(C), Ctype,
            ldc, sC, batch, compute, algo)

    def sgemm_strided_batched(self, transa, transb, m, n, k, alpha, A, lda, sA, B, ldb, sB,
                              beta, C, ldc, sC, batch) -> int:
        self._keep.clear()
        return self.lib.cublasSgemmStridedBatched(
            self.h, transa, transb, m, n, k, self._scalar(alpha, False), _ptr(A), lda, sA,
            _ptr(B), ldb, sB, self._scalar(beta, False), _ptr(C), ldc, sC, batch)

    def hgemm(self, transa, transb, m, n, k, alpha_bits: int, A, lda, B, ldb, beta_bits: int,
              C, ldc) -> int:
        a = ctypes.c_uint16(alpha_bits)
        b = ctypes.c_uint16(beta_bits)
        return self.lib.cublasHgemm(self.h, transa, transb, m, n, k, ctypes.byref(a), _ptr(A),
                                    lda, _ptr(B), ldb, ctypes.byref(b), _ptr(C), ldc)


def device_error() -> int:
    """Reads and clears the library's device error word (synchronises)."""
    return load().zlift_device_error()


def launch_count() -> int:
    return int(load().zlift_launch_count())
