"""CPU: the C ABI boundary.  The libraries load, export every entry point
that include/*.h declares (as zLift's build checks its exports,
zblas/build.sh:48), and answer host-side argument errors with the
reference's status codes before touching the GPU."""
import ctypes
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    names = set()
    for h in ("zlift_cublas.h", "zlift_cublaslt.h", "zlift_attention.h", "zlift_partition.h"):
        lines = open(os.path.join(ROOT, "include", h)).read().splitlines()
        src = "\n".join(l for l in lines if not l.lstrip().startswith("#"))
        for m in re.finditer(r"ZLIFT_API\s+[^;(]*?\b(\w+)\s*\(", src):
            names.add(m.group(1))
    return names


def _exported(path):
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True,
                         check=True).stdout
    return {line.split()[-1] for line in out.splitlines() if " T " in line}


def test_every_declared_symbol_is_exported(built_lib):
    import zlift_b200
    declared = _declared()
    assert len(declared) >= 35 and "__attribute__" not in declared
    missing = declared - _exported(zlift_b200.LIBCUBLAS)
    assert not missing, f"declared but not exported: {sorted(missing)}"


def test_library_names_and_soname(built_lib):
    import zlift_b200
    lib_dir = os.path.dirname(zlift_b200.LIBCUBLAS)
    for name in ("libcublas.so.13", "libcublas.so", "libcudnn.so.9", "libcudnn.so"):
        assert os.path.exists(os.path.join(lib_dir, name)), name
    out = subprocess.run(["readelf", "-d", zlift_b200.LIBCUBLAS], capture_output=True,
                         text=True).stdout
    assert "libcublas.so.13" in out and "SONAME" in out
    dnn = _exported(zlift_b200.LIBCUDNN)
    assert {"zblas_gpu_flash_f16", "zblas_gpu_fmha_f16"} <= dnn


def test_cudnn_library_loads_by_name(built_lib):
    """libcudnn.so.9 carries the real cuDNN soname (it is a drop-in), so a
    process that loads it before PyTorch would hand it to PyTorch's own
    cuDNN lookup.  Load it in a child process of its own."""
    import sys
    import zlift_b200
    code = ("import ctypes, os; l = ctypes.CDLL(%r, mode=os.RTLD_LOCAL); "
            "l.zblas_gpu_flash_f16.restype = ctypes.c_int; "
            "assert l.cudnnGetVersion() == 90000; "
            "assert l.zblas_gpu_flash_f16(None, 0, 1) == 1; print('ok')") % zlift_b200.LIBCUDNN
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode == 0 and "ok" in r.stdout, r.stderr


def test_handle_lifecycle_and_modes(built_lib):
    lib = built_lib
    h = ctypes.c_void_p()
    assert lib.cublasCreate_v2(ctypes.byref(h)) == 0
    v = ctypes.c_int()
    assert lib.cublasGetVersion_v2(h, ctypes.byref(v)) == 0 and v.value == 130000
    assert lib.cublasSetPointerMode_v2(h, 1) == 0
    assert lib.cublasGetPointerMode_v2(h, ctypes.byref(v)) == 0 and v.value == 1
    assert lib.cublasSetPointerMode_v2(h, 5) == 7
    assert lib.cublasSetMathMode(h, 3) == 0
    assert lib.cublasGetMathMode(h, ctypes.byref(v)) == 0 and v.value == 3
    s = ctypes.c_void_p()
    assert lib.cublasSetStream_v2(h, ctypes.c_void_p(0x1234)) == 0
    assert lib.cublasGetStream_v2(h, ctypes.byref(s)) == 0 and s.value == 0x1234
    assert lib.cublasDestroy_v2(h) == 0


def test_status_names(built_lib):
    lib = built_lib
    assert lib.cublasGetStatusName(0) == b"CUBLAS_STATUS_SUCCESS"
    assert lib.cublasGetStatusName(15) == b"CUBLAS_STATUS_NOT_SUPPORTED"
    assert lib.cublasGetStatusName(99) == b"CUBLAS_STATUS_INTERNAL_ERROR"


def test_null_handle_is_not_initialized(built_lib):
    lib = built_lib
    one = ctypes.c_float(1.0)
    assert lib.cublasSgemm_v2(None, 0, 0, 4, 4, 4, ctypes.byref(one), None, 4, None, 4,
                              ctypes.byref(one), None, 4) == 1
    assert lib.cublasGemmEx(None, 0, 0, 4, 4, 4, ctypes.byref(one), None, 2, 4, None, 2, 4,
                            ctypes.byref(one), None, 2, 4, 68, 0) == 1
    assert lib.cublasSetStream_v2(None, None) == 1


@pytest.fixture
def handle(built_lib):
    h = ctypes.c_void_p()
    assert built_lib.cublasCreate_v2(ctypes.byref(h)) == 0
    yield h
    built_lib.cublasDestroy_v2(h)


def _gemm_ex(lib, h, *, ta=0, tb=0, m=8, n=8, k=8, At=2, Bt=2, Ct=2, lda=8, ldb=8, ldc=8,
             compute=68, scalars=True, C=1):
    one = ctypes.c_float(1.0)
    al = ctypes.byref(one) if scalars else None
    return lib.cublasGemmEx(h, ta, tb, m, n, k, al, 16, At, lda, 16, Bt, ldb, al,
                            C and 16, Ct, ldc, compute, 0)


def test_argument_errors(built_lib, handle):
    lib = built_lib
    assert _gemm_ex(lib, handle, m=-1) == 7
    assert _gemm_ex(lib, handle, ta=5) == 7
    assert _gemm_ex(lib, handle, lda=4) == 7            # lda < m for op N
    assert _gemm_ex(lib, handle, ta=1, k=16, lda=8) == 7  # lda < k for op T
    assert _gemm_ex(lib, handle, ldc=7) == 7
    assert _gemm_ex(lib, handle, scalars=False) == 7
    assert _gemm_ex(lib, handle, C=0) == 7


def test_unsupported_types(built_lib, handle):
    lib = built_lib
    assert _gemm_ex(lib, handle, compute=77) == 15
    assert _gemm_ex(lib, handle, At=2, Bt=14) == 15     # mixed fp16 / bf16
    assert _gemm_ex(lib, handle, At=14, Bt=14, Ct=2) == 15
    assert _gemm_ex(lib, handle, At=3, Bt=3, Ct=10, compute=68) == 15   # int8 needs 32I
    assert _gemm_ex(lib, handle, At=3, Bt=3, Ct=0, compute=72) == 15


def test_empty_problems_succeed_without_a_gpu(built_lib, handle):
    lib = built_lib
    assert _gemm_ex(lib, handle, m=0) == 0
    assert _gemm_ex(lib, handle, n=0) == 0
    one = ctypes.c_float(1.0)
    assert lib.cublasGemmStridedBatchedEx(handle, 0, 0, 8, 8, 8, ctypes.byref(one), 16, 2, 8,
                                          64, 16, 2, 8, 64, ctypes.byref(one), 16, 2, 8, 64,
                                          0, 68, 0) == 0
    assert lib.cublasGemmStridedBatchedEx(handle, 0, 0, 8, 8, 8, ctypes.byref(one), 16, 2, 8,
                                          64, 16, 2, 8, 64, ctypes.byref(one), 16, 2, 8, 64,
                                          -1, 68, 0) == 7


def test_attention_declines_on_host(built_lib):
    """Blocks the kernel cannot serve are declined (1) before any launch."""
    from zlift_b200 import attention
    blk = attention.FlashBlock()
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 448, 1, None) == 1       # null operands
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 100, 1, None) == 1       # short block
    p = blk.p
    p.q_ptr = p.k_ptr = p.v_ptr = p.o_ptr = 0x1000
    p.b, p.h, p.h_k, p.h_h_k_ratio, p.seqlen_q, p.seqlen_k, p.d = 1, 2, 2, 1, 128, 128, 128
    p.p_dropout, p.p_dropout_in_uint8_t, p.rp_dropout = 1.0, 255, 1.0
    p.window_size_left = p.window_size_right = -1
    blk.is_bf16 = 1
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 448, 0, None) == 1       # dtype disagrees
    p.p_dropout = 0.9
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 448, 1, None) == 1       # dropout
    p.p_dropout = 1.0
    p.h_h_k_ratio = 3
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 448, 1, None) == 1       # head grouping
    p.h_h_k_ratio = 1
    p.d = 96
    assert built_lib.zlift_flash_fwd(ctypes.byref(blk), 448, 1, None) == 1       # head_dim 96
    fp = attention.FmhaParams()
    assert built_lib.zlift_fmha_fwd(ctypes.byref(fp), ctypes.sizeof(fp), 1, None) == 1


def test_noalloc_rejects_before_launch(built_lib, handle):
    one = ctypes.c_float(1.0)
    assert built_lib.zlift_sgemm_noalloc(None, 0, 0, 4, 4, 4, ctypes.byref(one), None, 4, None,
                                         4, ctypes.byref(one), None, 4) == 1
    assert built_lib.zlift_sgemm_noalloc(handle, 0, 0, 4096, 4096, 4096, ctypes.byref(one), 16,
                                         4096, 16, 4096, ctypes.byref(one), 16, 4096) == 7
