// cublas_api.cu -- the exported cuBLAS-style C ABI (see include/zlift_cublas.h).
//
// Host-side mirror of zLift's zblas/zblas.c: the same handle/stream/mode
// calls and the same GEMM entry points, argument conventions and status
// codes.  Every GEMM becomes one asynchronous launch on the handle's stream
// (tensor-core kernel, or the general CUDA-core kernel for layouts TMA
// cannot describe).  Nothing here runs arithmetic on the host.
#include "gemm.h"

#include "../../include/zlift_cublas.h"

#include <cuda_fp16.h>

#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <new>

namespace zl {

namespace {
std::atomic<unsigned long long> g_launches{0};
}

void note_launch(unsigned n) { g_launches.fetch_add(n, std::memory_order_relaxed); }
unsigned long long launch_count() { return g_launches.load(); }

bool tracing() {
    static int on = -1;
    if (on < 0) on = getenv("ZBLAS_TRACE") != nullptr;
    return on != 0;
}

static void trace(const char* fmt, ...) {
    if (!tracing()) return;
    va_list ap;
    va_start(ap, fmt);
    fprintf(stderr, "[zblas] ");
    vfprintf(stderr, fmt, ap);
    fprintf(stderr, "\n");
    va_end(ap);
}

// The state a cuBLAS handle carries (zblas/zblas.c:20-24), plus the
// scratch the fp32 path needs for its tf32 planes.
struct Handle {
    unsigned magic = 0x7a626c73;     // "zbls"
    cudaStream_t stream = nullptr;
    int pointer_mode = CUBLAS_POINTER_MODE_HOST;
    int math_mode = CUBLAS_DEFAULT_MATH;
    int device = 0;
    int sm_target = 0;
    void* user_ws = nullptr;         // cublasSetWorkspace_v2
    size_t user_ws_bytes = 0;
    void* scratch = nullptr;         // library-owned, grown on demand
    size_t scratch_bytes = 0;
    std::mutex mu;
};

static Handle* as_handle(cublasHandle_t h) {
    Handle* x = static_cast<Handle*>(h);
    return (x && x->magic == 0x7a626c73) ? x : nullptr;
}

// Device scratch of at least `bytes`: the user workspace if large enough,
// else a library allocation kept on the handle.  Freeing an old, smaller
// allocation waits for the device (cudaFree), as cuBLAS does when it grows
// its own workspace.
static void* handle_scratch(Handle* h, size_t bytes) {
    if (h->user_ws && h->user_ws_bytes >= bytes) return h->user_ws;
    if (h->scratch_bytes >= bytes) return h->scratch;
    if (h->scratch) cudaFree(h->scratch);
    h->scratch = nullptr;
    h->scratch_bytes = 0;
    void* p = nullptr;
    if (cudaMalloc(&p, bytes) != cudaSuccess) {
        cudaGetLastError();
        return nullptr;
    }
    h->scratch = p;
    h->scratch_bytes = bytes;
    return p;
}

static int elem_size(int t) {
    switch (t) {
    case kR16F: case kR16BF: return 2;
    case kR8I: return 1;
    default: return 4;
    }
}

static cublasStatus_t map_launch(int rc) {
    if (rc == 0) return CUBLAS_STATUS_SUCCESS;
    cudaGetLastError();
    return CUBLAS_STATUS_EXECUTION_FAILED;
}

// Runs one validated GEMM description: tensor cores first, CUDA cores when
// the layout is outside what TMA can describe.
static cublasStatus_t run_gemm(Handle* h, GemmDesc& d) {
    cudaStream_t s = h->stream;
    if (d.m == 0 || d.n == 0 || d.batch == 0) return CUBLAS_STATUS_SUCCESS;
    if (d.k == 0) return map_launch(gemm_simt(d, s));   // C = beta*C
    if (d.kind == Kind::TF32X3 || d.kind == Kind::TF32) {
        // tf32 planes of A and B in scratch, K-major with 16-byte rows:
        // hi = rn(x) (and lo = rn(x - hi) for the 3-product form).  The
        // reference splits into bf16 planes instead (split_to_bf16,
        // zblas_gpu.cpp:219-265).
        const bool two = d.kind == Kind::TF32X3;
        const long long kp = ((long long)d.k + 3) & ~3ll;
        auto up = [](long long e) { return (e + 63) & ~63ll; };   // 256-byte aligned planes
        const long long ea = up((long long)d.m * kp * d.batch);
        const long long eb = up((long long)d.n * kp * d.batch);
        const size_t bytes = (size_t)((two ? 2 : 1) * (ea + eb)) * sizeof(float);
        std::lock_guard<std::mutex> lock(h->mu);
        float* base = static_cast<float*>(handle_scratch(h, bytes));
        if (!base) return CUBLAS_STATUS_NOT_INITIALIZED;   // allocation failure (zblas.c:333-337)
        float* a_hi = base;
        float* b_hi = a_hi + ea;
        float* a_lo = two ? b_hi + eb : nullptr;
        float* b_lo = two ? a_lo + ea : nullptr;
        // op(A)(i,l) is A[l + i*lda] (K contiguous) for transa != N
        int rc = split_tf32(static_cast<const float*>(d.A), d.transa != 0, d.m, d.k, d.lda,
                            d.strideA, d.batch, kp, a_hi, a_lo, s);
        // op(B)(l,j) is B[l + j*ldb] (K contiguous) for transb == N
        if (rc == 0)
            rc = split_tf32(static_cast<const float*>(d.B), d.transb == 0, d.n, d.k, d.ldb,
                            d.strideB, d.batch, kp, b_hi, b_lo, s);
        if (rc) return map_launch(rc);
        GemmDesc e = d;
        e.transa = 1;               // planes are K-major: op(A) = A^T of a k x m matrix
        e.transb = 0;
        e.A = a_hi; e.B = b_hi;
        e.lda = kp; e.ldb = kp;
        e.strideA = (long long)d.m * kp;
        e.strideB = (long long)d.n * kp;
        e.A_hi = a_hi; e.A_lo = a_lo; e.B_hi = b_hi; e.B_lo = b_lo;
        rc = gemm_tc(e, s);
        if (rc == 1) rc = gemm_simt(d, s);   // plain fp32 on CUDA cores
        return map_launch(rc);
    }
    int rc = gemm_tc(d, s);
    if (rc == 1) rc = gemm_simt(d, s);
    return map_launch(rc);
}

// Shared argument checks of every GEMM entry (the reference passes these
// straight to cblas, which would reject them with an error message).
static cublasStatus_t check_dims(int transa, int transb, int m, int n, int k,
                                 long long lda, long long ldb, long long ldc) {
    if (transa < 0 || transa > 2 || transb < 0 || transb > 2) return CUBLAS_STATUS_INVALID_VALUE;
    if (m < 0 || n < 0 || k < 0) return CUBLAS_STATUS_INVALID_VALUE;
    const long long ra = transa == CUBLAS_OP_N ? m : k;
    const long long rb = transb == CUBLAS_OP_N ? k : n;
    if (lda < (ra > 1 ? ra : 1) || ldb < (rb > 1 ? rb : 1) || ldc < (m > 1 ? m : 1))
        return CUBLAS_STATUS_INVALID_VALUE;
    return CUBLAS_STATUS_SUCCESS;
}

// Reads the scalars according to the pointer mode.  32F: float; 32I: int32.
static cublasStatus_t set_scalars(Handle* h, GemmDesc& d, const void* alpha,
                                  const void* beta, bool integer) {
    if (!alpha || !beta) return CUBLAS_STATUS_INVALID_VALUE;
    d.alpha_dev = d.beta_dev = nullptr;
    d.alpha = d.beta = 0.f;
    d.ialpha = d.ibeta = 0;
    if (h->pointer_mode == CUBLAS_POINTER_MODE_DEVICE) {
        d.alpha_dev = alpha;
        d.beta_dev = beta;
    } else if (integer) {
        d.ialpha = *static_cast<const int32_t*>(alpha);
        d.ibeta = *static_cast<const int32_t*>(beta);
    } else {
        d.alpha = *static_cast<const float*>(alpha);
        d.beta = *static_cast<const float*>(beta);
    }
    return CUBLAS_STATUS_SUCCESS;
}

// Type/compute dispatch of cublasGemmEx (zblas/zblas.c:357-391) for one
// (possibly batched) call.
static cublasStatus_t gemm_ex(Handle* h, int transa, int transb, int m, int n, int k,
                              const void* alpha, const void* A, int Atype, int lda,
                              long long sA, const void* B, int Btype, int ldb,
                              long long sB, const void* beta, void* C, int Ctype,
                              int ldc, long long sC, int batch, int computeType) {
    cublasStatus_t st = check_dims(transa, transb, m, n, k, lda, ldb, ldc);
    if (st) return st;
    if (batch < 0) return CUBLAS_STATUS_INVALID_VALUE;
    GemmDesc d{};
    d.transa = transa == CUBLAS_OP_N ? 0 : 1;
    d.transb = transb == CUBLAS_OP_N ? 0 : 1;
    d.m = m; d.n = n; d.k = k; d.batch = batch;
    d.A = A; d.lda = lda; d.strideA = sA; d.Atype = Atype;
    d.B = B; d.ldb = ldb; d.strideB = sB; d.Btype = Btype;
    d.C = C; d.ldc = ldc; d.strideC = sC; d.Ctype = Ctype;
    bool integer = false;
    if (Atype == kR8I && Btype == kR8I && Ctype == kR32I &&
        (computeType == CUBLAS_COMPUTE_32I || computeType == kR32I)) {
        d.kind = Kind::I8;
        integer = true;
    } else {
        if (computeType != kR32F && computeType != CUBLAS_COMPUTE_32F)
            return CUBLAS_STATUS_NOT_SUPPORTED;
        if (Atype == kR32F && Btype == kR32F && Ctype == kR32F) {
            d.kind = h->math_mode == CUBLAS_TF32_TENSOR_OP_MATH ? Kind::TF32 : Kind::TF32X3;
        } else if (Atype == kR16BF && Btype == kR16BF && (Ctype == kR16BF || Ctype == kR32F)) {
            d.kind = Kind::BF16;
        } else if (Atype == kR16F && Btype == kR16F && (Ctype == kR16F || Ctype == kR32F)) {
            d.kind = Kind::F16;
        } else {
            return CUBLAS_STATUS_NOT_SUPPORTED;
        }
    }
    if (m == 0 || n == 0 || batch == 0) return CUBLAS_STATUS_SUCCESS;
    if (!C || (k > 0 && (!A || !B))) return CUBLAS_STATUS_INVALID_VALUE;
    st = set_scalars(h, d, alpha, beta, integer);
    if (st) return st;
    trace("gemm kind=%d %dx%dx%d batch=%d ta=%d tb=%d lda=%d ldb=%d ldc=%d", (int)d.kind, m, n,
          k, batch, transa, transb, lda, ldb, ldc);
    return run_gemm(h, d);
}

}  // namespace zl

using namespace zl;

extern "C" {

cublasStatus_t cublasCreate_v2(cublasHandle_t* handle) {
    if (!handle) return CUBLAS_STATUS_INVALID_VALUE;
    Handle* h = new (std::nothrow) Handle();
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    cudaGetDevice(&h->device);
    *handle = h;
    trace("create");
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasDestroy_v2(cublasHandle_t handle) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (h->scratch) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(h->device);
        cudaFree(h->scratch);
        cudaSetDevice(cur);
    }
    h->magic = 0;
    delete h;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetVersion_v2(cublasHandle_t, int* version) {
    if (!version) return CUBLAS_STATUS_INVALID_VALUE;
    *version = 130000;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, void* stream) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    h->stream = static_cast<cudaStream_t>(stream);
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, void** stream) {
    Handle* h = as_handle(handle);
    if (!h || !stream) return CUBLAS_STATUS_INVALID_VALUE;
    *stream = h->stream;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, int mode) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (mode != CUBLAS_POINTER_MODE_HOST && mode != CUBLAS_POINTER_MODE_DEVICE)
        return CUBLAS_STATUS_INVALID_VALUE;
    h->pointer_mode = mode;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, int* mode) {
    Handle* h = as_handle(handle);
    if (!h || !mode) return CUBLAS_STATUS_INVALID_VALUE;
    *mode = h->pointer_mode;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetMathMode(cublasHandle_t handle, int mode) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    h->math_mode = mode;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetMathMode(cublasHandle_t handle, int* mode) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (!mode) return CUBLAS_STATUS_INVALID_VALUE;
    *mode = h->math_mode;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetWorkspace_v2(cublasHandle_t handle, void* workspace, size_t bytes) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    std::lock_guard<std::mutex> lock(h->mu);
    h->user_ws = workspace;
    h->user_ws_bytes = workspace ? bytes : 0;
    trace("setWorkspace %zu", bytes);
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasSetSmCountTarget(cublasHandle_t handle, int count) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (count < 0) return CUBLAS_STATUS_INVALID_VALUE;
    h->sm_target = count;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasGetSmCountTarget(cublasHandle_t handle, int* count) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (count) *count = h->sm_target;
    return CUBLAS_STATUS_SUCCESS;
}

const char* cublasGetStatusName(cublasStatus_t s) {
    switch (s) {
    case CUBLAS_STATUS_SUCCESS: return "CUBLAS_STATUS_SUCCESS";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "CUBLAS_STATUS_NOT_INITIALIZED";
    case CUBLAS_STATUS_INVALID_VALUE: return "CUBLAS_STATUS_INVALID_VALUE";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "CUBLAS_STATUS_EXECUTION_FAILED";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "CUBLAS_STATUS_NOT_SUPPORTED";
    default: return "CUBLAS_STATUS_INTERNAL_ERROR";
    }
}

const char* cublasGetStatusString(cublasStatus_t s) {
    switch (s) {
    case CUBLAS_STATUS_SUCCESS: return "success";
    case CUBLAS_STATUS_NOT_INITIALIZED: return "the library was not initialized";
    case CUBLAS_STATUS_INVALID_VALUE: return "an invalid numeric value was used as an argument";
    case CUBLAS_STATUS_EXECUTION_FAILED: return "the GPU program failed to execute";
    case CUBLAS_STATUS_NOT_SUPPORTED: return "the functionality requested is not supported";
    default: return "an internal operation failed";
    }
}

cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, int transa, int transb, int m, int n,
                              int k, const float* alpha, const float* A, int lda,
                              const float* B, int ldb, const float* beta, float* C, int ldc) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    return gemm_ex(h, transa, transb, m, n, k, alpha, A, kR32F, lda, 0, B, kR32F, ldb, 0, beta,
                   C, kR32F, ldc, 0, 1, CUBLAS_COMPUTE_32F);
}

cublasStatus_t cublasGemmEx(cublasHandle_t handle, int transa, int transb, int m, int n, int k,
                            const void* alpha, const void* A, int Atype, int lda,
                            const void* B, int Btype, int ldb, const void* beta, void* C,
                            int Ctype, int ldc, int computeType, int algo) {
    (void)algo;
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    return gemm_ex(h, transa, transb, m, n, k, alpha, A, Atype, lda, 0, B, Btype, ldb, 0, beta,
                   C, Ctype, ldc, 0, 1, computeType);
}

cublasStatus_t cublasGemmStridedBatchedEx(cublasHandle_t handle, int transa, int transb, int m,
                                          int n, int k, const void* alpha, const void* A,
                                          int Atype, int lda, long long strideA, const void* B,
                                          int Btype, int ldb, long long strideB,
                                          const void* beta, void* C, int Ctype, int ldc,
                                          long long strideC, int batchCount, int computeType,
                                          int algo) {
    (void)algo;
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    return gemm_ex(h, transa, transb, m, n, k, alpha, A, Atype, lda, strideA, B, Btype, ldb,
                   strideB, beta, C, Ctype, ldc, strideC, batchCount, computeType);
}

cublasStatus_t cublasSgemmStridedBatched(cublasHandle_t handle, int transa, int transb, int m,
                                         int n, int k, const float* alpha, const float* A,
                                         int lda, long long strideA, const float* B, int ldb,
                                         long long strideB, const float* beta, float* C,
                                         int ldc, long long strideC, int batchCount) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    return gemm_ex(h, transa, transb, m, n, k, alpha, A, kR32F, lda, strideA, B, kR32F, ldb,
                   strideB, beta, C, kR32F, ldc, strideC, batchCount, CUBLAS_COMPUTE_32F);
}

cublasStatus_t cublasSgemmEx(cublasHandle_t handle, int transa, int transb, int m, int n, int k,
                             const float* alpha, const void* A, int Atype, int lda,
                             const void* B, int Btype, int ldb, const float* beta, void* C,
                             int Ctype, int ldc) {
    return cublasGemmEx(handle, transa, transb, m, n, k, alpha, A, Atype, lda, B, Btype, ldb,
                        beta, C, Ctype, ldc, kR32F, 0);
}

cublasStatus_t cublasHgemm(cublasHandle_t handle, int transa, int transb, int m, int n, int k,
                           const unsigned short* alpha, const unsigned short* A, int lda,
                           const unsigned short* B, int ldb, const unsigned short* beta,
                           unsigned short* C, int ldc) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    if (!alpha || !beta) return CUBLAS_STATUS_INVALID_VALUE;
    if (h->pointer_mode == CUBLAS_POINTER_MODE_DEVICE) {
        // fp16 scalars on the device: the kernels take fp32 scalars, so
        // this form is not offered (cuBLAS itself converts on the device).
        return CUBLAS_STATUS_NOT_SUPPORTED;
    }
    __half_raw ra, rb;
    ra.x = *alpha;
    rb.x = *beta;
    const float fa = __half2float(__half(ra)), fb = __half2float(__half(rb));
    return gemm_ex(h, transa, transb, m, n, k, &fa, A, kR16F, lda, 0, B, kR16F, ldb, 0, &fb, C,
                   kR16F, ldc, 0, 1, CUBLAS_COMPUTE_32F);
}

int zlift_device_error(void) {
    cudaDeviceSynchronize();
    int e = gemm_tc_error(true);
    int e2 = gemm_simt_error(true);
    int e3 = fmha_error(true);
    return e ? e : (e2 ? e2 : e3);
}

unsigned long long zlift_launch_count(void) { return launch_count(); }

}  // extern "C"
