"""zlift_b200 -- zLift's GEMM and fused-attention hot path, B200-native.

The product is the pair of native libraries under ``zlift_b200/lib``:
``libcublas.so.13`` (cuBLAS-style C ABI + every CUDA kernel) and
``libcudnn.so.9`` (the attention entry points under the cuDNN name).  This
package only loads them through ctypes and exposes the same calls to
Python; it does no arithmetic itself.  If the libraries are missing, every
entry raises -- there is no fallback.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_DIR = os.path.join(HERE, "lib")
LIBCUBLAS = os.path.join(LIB_DIR, "libcublas.so.13")
LIBCUDNN = os.path.join(LIB_DIR, "libcudnn.so.9")

_lib = None

c_int, c_uint, c_float, c_void_p = ctypes.c_int, ctypes.c_uint, ctypes.c_float, ctypes.c_void_p
c_ll, c_size_t = ctypes.c_longlong, ctypes.c_size_t

# (name, restype, argtypes) of every C entry point declared in include/*.h
SIGNATURES = [
    ("cublasCreate_v2", c_int, [ctypes.POINTER(c_void_p)]),
    ("cublasDestroy_v2", c_int, [c_void_p]),
    ("cublasGetVersion_v2", c_int, [c_void_p, ctypes.POINTER(c_int)]),
    ("cublasSetStream_v2", c_int, [c_void_p, c_void_p]),
    ("cublasGetStream_v2", c_int, [c_void_p, ctypes.POINTER(c_void_p)]),
    ("cublasSetPointerMode_v2", c_int, [c_void_p, c_int]),
    ("cublasGetPointerMode_v2", c_int, [c_void_p, ctypes.POINTER(c_int)]),
    ("cublasSetMathMode", c_int, [c_void_p, c_int]),
    ("cublasGetMathMode", c_int, [c_void_p, ctypes.POINTER(c_int)]),
    ("cublasSetWorkspace_v2", c_int, [c_void_p, c_void_p, c_size_t]),
    ("cublasSetSmCountTarget", c_int, [c_void_p, c_int]),
    ("cublasGetSmCountTarget", c_int, [c_void_p, ctypes.POINTER(c_int)]),
    ("cublasGetStatusName", ctypes.c_char_p, [c_int]),
    ("cublasGetStatusString", ctypes.c_char_p, [c_int]),
    ("cublasSgemm_v2", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                               c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int]),
    ("cublasDgemm_v2", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                               c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int]),
    ("cublasGemmEx", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                             c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p,
                             c_void_p, c_int, c_int, c_int, c_int]),
    ("cublasGemmStridedBatchedEx", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int,
                                           c_void_p, c_void_p, c_int, c_int, c_ll,
                                           c_void_p, c_int, c_int, c_ll, c_void_p,
                                           c_void_p, c_int, c_int, c_ll, c_int, c_int, c_int]),
    ("cublasSgemmStridedBatched", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int,
                                          c_void_p, c_void_p, c_int, c_ll, c_void_p, c_int,
                                          c_ll, c_void_p, c_void_p, c_int, c_ll, c_int]),
    ("cublasSgemmEx", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                              c_void_p, c_int, c_int, c_void_p, c_int, c_int, c_void_p,
                              c_void_p, c_int, c_int]),
    ("cublasHgemm", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                            c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p, c_int]),
    ("zlift_sgemm_noalloc", c_int, [c_void_p, c_int, c_int, c_int, c_int, c_int, c_void_p,
                                    c_void_p, c_int, c_void_p, c_int, c_void_p, c_void_p,
                                    c_int]),
    ("zlift_device_error", c_int, []),
    ("zlift_launch_count", ctypes.c_ulonglong, []),
    ("zlift_set_wait_limit_ns", c_int, [ctypes.c_ulonglong]),
    ("zlift_get_wait_limit_ns", ctypes.c_ulonglong, []),
    ("zlift_wait_probe", c_int, [ctypes.c_ulonglong, c_void_p]),
    ("zblas_gpu_flash_f16", c_int, [c_void_p, c_uint, c_int]),
    ("zblas_gpu_fmha_f16", c_int, [c_void_p, c_uint, c_int]),
    ("zblas_attention_set_stream", None, [c_void_p]),
    ("zblas_attention_get_stream", c_void_p, []),
    ("zlift_flash_fwd", c_int, [c_void_p, c_uint, c_int, c_void_p]),
    ("zlift_fmha_fwd", c_int, [c_void_p, c_uint, c_int, c_void_p]),
    ("zlift_part_range", c_int, [c_ll, c_int, c_int, c_ll, ctypes.POINTER(c_ll),
                                 ctypes.POINTER(c_ll)]),
    ("zlift_part_unique_id", c_int, [c_void_p]),
    ("zlift_part_comm_init", c_int, [ctypes.POINTER(c_void_p), c_int, c_int, c_void_p]),
    ("zlift_part_comm_destroy", c_int, [c_void_p]),
    ("zlift_part_comm_wait", c_int, [c_void_p, c_void_p, c_int]),
    ("zlift_part_gemm_strided_batched_ex", c_int, [c_void_p, c_ll, c_ll, c_int, c_int, c_int,
                                                   c_int, c_int, c_void_p, c_void_p, c_int,
                                                   c_int, c_ll, c_void_p, c_int, c_int, c_ll,
                                                   c_void_p, c_void_p, c_int, c_int, c_ll,
                                                   c_int]),
    ("zlift_part_gemm_ex_nsplit", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int, c_int,
                                          c_int, c_int, c_void_p, c_void_p, c_int, c_int,
                                          c_void_p, c_int, c_int, c_void_p, c_void_p, c_int,
                                          c_int]),
    ("zlift_part_nsplit_cols", c_int, [c_ll, c_int, c_int, c_int, c_int, ctypes.POINTER(c_ll),
                                       ctypes.POINTER(c_ll)]),
    ("zlift_part_gemm_ex_nsplit_overlap", c_int, [c_void_p, c_void_p, c_int, c_int, c_int, c_int,
                                                  c_int, c_int, c_int, c_int, c_void_p, c_void_p,
                                                  c_int, c_int, c_void_p, c_int, c_int, c_void_p,
                                                  c_void_p, c_int, c_int]),
    ("zlift_part_register_peer_buffer", c_int, [c_void_p, c_int, c_int, c_void_p, c_size_t]),
    ("zlift_part_unregister_peer_buffer", c_int, [c_void_p, c_void_p]),
    ("zlift_part_flash_fwd", c_int, [c_void_p, c_uint, c_int, c_ll, c_ll, c_void_p]),
]


def load(path: str | None = None) -> ctypes.CDLL:
    """Loads libcublas.so.13 (RTLD_LOCAL, so it never interposes on the
    cuBLAS that PyTorch itself uses) and declares every entry point."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = path or LIBCUBLAS
    if not os.path.exists(p):
        raise ImportError(f"{p} is not built; run `python -m zlift_b200.build`")
    lib = ctypes.CDLL(p, mode=os.RTLD_LOCAL | os.RTLD_NOW)
    for name, res, args in SIGNATURES:
        fn = getattr(lib, name, None)
        if fn is None:
            continue
        fn.restype = res
        fn.argtypes = args
    if path is None:
        _lib = lib
    return lib


from .blas import Handle, GemmError  # noqa: E402
from .attention import flash_forward, fmha_forward, FlashParams, FmhaParams  # noqa: E402

__all__ = ["load", "Handle", "GemmError", "flash_forward", "fmha_forward",
           "FlashParams", "FmhaParams", "LIBCUBLAS", "LIBCUDNN"]
