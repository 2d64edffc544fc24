// cublas_api.cu -- the exported cuBLAS-style C ABI (see include/zlift_cublas.h).
//
// Host-side mirror of zLift's zblas/zblas.c: the same handle/stream/mode
// calls and the same GEMM entry points, argument conventions and status
// codes.  Every GEMM becomes one asynchronous launch on the handle's stream
// (tensor-core kernel, or the general CUDA-core kernel for layouts TMA
// cannot describe).  Nothing here runs arithmetic on the host.
#include "gemm.h"

#include "../../include/zlift_cublas.h"
#include "../../include/zlift_cublaslt.h"

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
    // K-split tail workspaces (counters, then partial sums), one per stream
    // the handle has launched split GEMMs on, so that split launches on
    // different streams never share counters
    struct SplitWs {
        cudaStream_t stream = nullptr;
        void* ws = nullptr;
        unsigned long long epoch = 0;
    };
    static constexpr int kSplitStreams = 4;
    SplitWs split[kSplitStreams];
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

// Workspace of the tensor-core kernel's K-split tail (GemmDesc::split_work):
// tile counters, then partial sums; the largest split needs 2 * 74 parts of
// 128 x 256 fp32 values (18.9 MB).  One workspace per stream (up to
// kSplitStreams streams per handle; calls on further streams run without a
// split), allocated on the first GEMM on that stream, except inside a
// stream capture, where the GEMM goes without it.  Each launch gets the
// next epoch of its stream's workspace.  Called with h->mu held.
constexpr size_t kSplitCounterBytes = 4096;
constexpr size_t kSplitWorkBytes = 20u << 20;

static void attach_split_ws(Handle* h, GemmDesc& d, cudaStream_t s) {
    Handle::SplitWs* w = nullptr;
    for (auto& x : h->split)
        if (x.ws && x.stream == s) w = &x;
    if (!w) {
        Handle::SplitWs* slot = nullptr;
        for (auto& x : h->split)
            if (!x.ws && !slot) slot = &x;
        if (!slot) return;
        cudaStreamCaptureStatus cs = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(s, &cs) != cudaSuccess || cs != cudaStreamCaptureStatusNone) {
            cudaGetLastError();
            return;
        }
        void* p = nullptr;
        if (cudaMalloc(&p, kSplitCounterBytes + kSplitWorkBytes) != cudaSuccess) {
            cudaGetLastError();
            return;
        }
        if (cudaMemsetAsync(p, 0, kSplitCounterBytes, s) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(p);
            return;
        }
        slot->stream = s;
        slot->ws = p;
        slot->epoch = 0;
        w = slot;
    }
    d.split_counters = static_cast<unsigned long long*>(w->ws);
    d.split_work = reinterpret_cast<uint32_t*>(static_cast<char*>(w->ws) + kSplitCounterBytes);
    d.split_work_bytes = kSplitWorkBytes;
    d.split_epoch = ++w->epoch;
}

// Runs one validated GEMM description: tensor cores first, CUDA cores when
// the layout is outside what TMA can describe.
static cublasStatus_t run_gemm(Handle* h, GemmDesc& d, cudaStream_t s) {
    if (d.m == 0 || d.n == 0 || d.batch == 0) return CUBLAS_STATUS_SUCCESS;
    d.sm_limit = h->sm_target;
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
        attach_split_ws(h, e, s);
        rc = gemm_tc(e, s);
        if (rc == 1) rc = gemm_simt(d, s);   // plain fp32 on CUDA cores
        return map_launch(rc);
    }
    std::lock_guard<std::mutex> lock(h->mu);
    attach_split_ws(h, d, s);
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
static cublasStatus_t set_scalars(int pointer_mode, GemmDesc& d, const void* alpha,
                                  const void* beta, bool integer) {
    if (!alpha || !beta) return CUBLAS_STATUS_INVALID_VALUE;
    d.alpha_dev = d.beta_dev = nullptr;
    d.alpha = d.beta = 0.f;
    d.ialpha = d.ibeta = 0;
    if (pointer_mode == CUBLAS_POINTER_MODE_DEVICE) {
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

// What cublasLtMatmul adds to a GEMM call: a fused epilogue, its own
// stream and its own pointer mode.
struct LtExtra {
    int epi;
    const void* bias;
    int bias_type;
    cudaStream_t stream;
    int pointer_mode;
    int scale_type;
};

// Type/compute dispatch of cublasGemmEx (zblas/zblas.c:357-391) for one
// (possibly batched) call.
static cublasStatus_t gemm_ex(Handle* h, int transa, int transb, int m, int n, int k,
                              const void* alpha, const void* A, int Atype, int lda,
                              long long sA, const void* B, int Btype, int ldb,
                              long long sB, const void* beta, void* C, int Ctype,
                              int ldc, long long sC, int batch, int computeType,
                              const LtExtra* lt = nullptr) {
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
    const bool compute_i = computeType == CUBLAS_COMPUTE_32I || computeType == kR32I;
    if (Atype == kR8I && Btype == kR8I && Ctype == kR32I && compute_i) {
        d.kind = Kind::I8;
        integer = true;
    } else if (lt && Atype == kR8I && Btype == kR8I && Ctype == kR8I && compute_i) {
        // cuBLASLt's int8 output: float alpha/beta (scale type 32F),
        // D = sat_s8(rne(alpha * acc + beta * C)) -- the requantising epilogue
        if (lt->scale_type != kR32F) return CUBLAS_STATUS_NOT_SUPPORTED;
        d.kind = Kind::I8;
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
    if (lt && lt->epi && d.kind == Kind::I8) return CUBLAS_STATUS_NOT_SUPPORTED;
    if (m == 0 || n == 0 || batch == 0) return CUBLAS_STATUS_SUCCESS;
    if (!C || (k > 0 && (!A || !B))) return CUBLAS_STATUS_INVALID_VALUE;
    st = set_scalars(lt ? lt->pointer_mode : h->pointer_mode, d, alpha, beta, integer);
    if (st) return st;
    if (lt) {
        d.epi = lt->epi;
        d.bias = lt->bias;
        d.bias_type = lt->bias_type;
    }
    trace("gemm kind=%d %dx%dx%d batch=%d ta=%d tb=%d lda=%d ldb=%d ldc=%d epi=%d", (int)d.kind,
          m, n, k, batch, transa, transb, lda, ldb, ldc, d.epi);
    return run_gemm(h, d, lt ? lt->stream : h->stream);
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
    bool any = h->scratch != nullptr;
    for (auto& x : h->split) any = any || x.ws;
    if (any) {
        int cur = 0;
        cudaGetDevice(&cur);
        cudaSetDevice(h->device);
        if (h->scratch) cudaFree(h->scratch);
        for (auto& x : h->split)
            if (x.ws) cudaFree(x.ws);
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

cublasStatus_t cublasDgemm_v2(cublasHandle_t handle, int transa, int transb, int m, int n,
                              int k, const double* alpha, const double* A, int lda,
                              const double* B, int ldb, const double* beta, double* C, int ldc) {
    Handle* h = as_handle(handle);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    cublasStatus_t st = check_dims(transa, transb, m, n, k, lda, ldb, ldc);
    if (st) return st;
    if (m == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
    if (!alpha || !beta || !C || (k > 0 && (!A || !B))) return CUBLAS_STATUS_INVALID_VALUE;
    const bool dev = h->pointer_mode == CUBLAS_POINTER_MODE_DEVICE;
    trace("dgemm %dx%dx%d ta=%d tb=%d", m, n, k, transa, transb);
    return map_launch(dgemm_simt(transa == CUBLAS_OP_N ? 0 : 1, transb == CUBLAS_OP_N ? 0 : 1, m,
                                 n, k, dev ? 0.0 : *alpha, dev ? 0.0 : *beta,
                                 dev ? alpha : nullptr, dev ? beta : nullptr, A, lda, B, ldb, C,
                                 ldc, h->stream));
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

// ---- cuBLASLt subset (zblas/zblas.c:512-711) ---------------------------

}  // extern "C"

namespace {

struct LtDesc {
    unsigned magic = 0x4c746465;    // "Ltde"
    int compute_type = 0, scale_type = 0, pointer_mode = 0;
    int transa = 0, transb = 0, epilogue = CUBLASLT_EPILOGUE_DEFAULT;
    const void* bias = nullptr;
};

struct LtLayout {
    unsigned magic = 0x4c746c61;    // "Ltla"
    int type = 0, order = CUBLASLT_ORDER_COL;
    long long rows = 0, cols = 0, ld = 0;
    int batch = 1;
    long long batch_stride = 0;
};

LtDesc* as_desc(void* p) {
    LtDesc* d = static_cast<LtDesc*>(p);
    return d && d->magic == 0x4c746465 ? d : nullptr;
}
LtLayout* as_layout(void* p) {
    LtLayout* l = static_cast<LtLayout*>(p);
    return l && l->magic == 0x4c746c61 ? l : nullptr;
}

template <typename T>
cublasStatus_t put(T& field, const void* buf, size_t bytes) {
    if (bytes < sizeof(T)) return CUBLAS_STATUS_INVALID_VALUE;
    std::memcpy(&field, buf, sizeof(T));
    return CUBLAS_STATUS_SUCCESS;
}

}  // namespace

extern "C" {

cublasStatus_t cublasLtCreate(cublasLtHandle_t* handle) { return cublasCreate_v2(handle); }
cublasStatus_t cublasLtDestroy(cublasLtHandle_t handle) { return cublasDestroy_v2(handle); }
cublasStatus_t cublasLtGetVersion(void) { return 130100; }

cublasStatus_t cublasLtMatmulDescCreate(void** desc, int computeType, int scaleType) {
    if (!desc) return CUBLAS_STATUS_INVALID_VALUE;
    LtDesc* d = new (std::nothrow) LtDesc();
    if (!d) return CUBLAS_STATUS_NOT_INITIALIZED;
    d->compute_type = computeType;
    d->scale_type = scaleType;
    *desc = d;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatmulDescDestroy(void* desc) {
    LtDesc* d = as_desc(desc);
    if (d) {
        d->magic = 0;
        delete d;
    }
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatmulDescSetAttribute(void* desc, int attr, const void* buf,
                                              size_t bytes) {
    LtDesc* d = as_desc(desc);
    if (!d || !buf) return CUBLAS_STATUS_INVALID_VALUE;
    switch (attr) {
    case CUBLASLT_MATMUL_DESC_COMPUTE_TYPE: return put(d->compute_type, buf, bytes);
    case CUBLASLT_MATMUL_DESC_SCALE_TYPE: return put(d->scale_type, buf, bytes);
    case CUBLASLT_MATMUL_DESC_POINTER_MODE: return put(d->pointer_mode, buf, bytes);
    case CUBLASLT_MATMUL_DESC_TRANSA: return put(d->transa, buf, bytes);
    case CUBLASLT_MATMUL_DESC_TRANSB: return put(d->transb, buf, bytes);
    case CUBLASLT_MATMUL_DESC_EPILOGUE: return put(d->epilogue, buf, bytes);
    case CUBLASLT_MATMUL_DESC_BIAS_POINTER: return put(d->bias, buf, bytes);
    default: return CUBLAS_STATUS_SUCCESS;   // accepted and ignored, as in zblas.c:563
    }
}

cublasStatus_t cublasLtMatmulDescGetAttribute(void* desc, int attr, void* buf, size_t bytes,
                                              size_t* written) {
    LtDesc* d = as_desc(desc);
    if (!d || !buf) return CUBLAS_STATUS_INVALID_VALUE;
    if (attr == CUBLASLT_MATMUL_DESC_BIAS_POINTER) {
        if (bytes < sizeof(void*)) return CUBLAS_STATUS_INVALID_VALUE;
        std::memcpy(buf, &d->bias, sizeof(void*));
        if (written) *written = sizeof(void*);
        return CUBLAS_STATUS_SUCCESS;
    }
    int v = attr == CUBLASLT_MATMUL_DESC_TRANSA ? d->transa
          : attr == CUBLASLT_MATMUL_DESC_TRANSB ? d->transb
          : attr == CUBLASLT_MATMUL_DESC_EPILOGUE ? d->epilogue
          : attr == CUBLASLT_MATMUL_DESC_COMPUTE_TYPE ? d->compute_type
          : attr == CUBLASLT_MATMUL_DESC_SCALE_TYPE ? d->scale_type
          : attr == CUBLASLT_MATMUL_DESC_POINTER_MODE ? d->pointer_mode : 0;
    if (bytes < sizeof v) return CUBLAS_STATUS_INVALID_VALUE;
    std::memcpy(buf, &v, sizeof v);
    if (written) *written = sizeof v;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatrixLayoutCreate(void** layout, int type, unsigned long long rows,
                                          unsigned long long cols, long long ld) {
    if (!layout) return CUBLAS_STATUS_INVALID_VALUE;
    LtLayout* l = new (std::nothrow) LtLayout();
    if (!l) return CUBLAS_STATUS_NOT_INITIALIZED;
    l->type = type;
    l->rows = (long long)rows;
    l->cols = (long long)cols;
    l->ld = ld;
    *layout = l;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatrixLayoutDestroy(void* layout) {
    LtLayout* l = as_layout(layout);
    if (l) {
        l->magic = 0;
        delete l;
    }
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatrixLayoutSetAttribute(void* layout, int attr, const void* buf,
                                                size_t bytes) {
    LtLayout* l = as_layout(layout);
    if (!l || !buf) return CUBLAS_STATUS_INVALID_VALUE;
    switch (attr) {
    case CUBLASLT_MATRIX_LAYOUT_TYPE: return put(l->type, buf, bytes);
    case CUBLASLT_MATRIX_LAYOUT_ORDER: return put(l->order, buf, bytes);
    case CUBLASLT_MATRIX_LAYOUT_ROWS: {
        unsigned long long v;
        cublasStatus_t st = put(v, buf, bytes);
        if (!st) l->rows = (long long)v;
        return st;
    }
    case CUBLASLT_MATRIX_LAYOUT_COLS: {
        unsigned long long v;
        cublasStatus_t st = put(v, buf, bytes);
        if (!st) l->cols = (long long)v;
        return st;
    }
    case CUBLASLT_MATRIX_LAYOUT_LD: return put(l->ld, buf, bytes);
    case CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT: return put(l->batch, buf, bytes);
    case CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET: return put(l->batch_stride, buf, bytes);
    default: return CUBLAS_STATUS_SUCCESS;
    }
}

cublasStatus_t cublasLtMatmulPreferenceCreate(void** pref) {
    if (!pref) return CUBLAS_STATUS_INVALID_VALUE;
    void* p = calloc(1, 8);
    if (!p) return CUBLAS_STATUS_NOT_INITIALIZED;
    *pref = p;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatmulPreferenceDestroy(void* pref) {
    free(pref);
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatmulPreferenceSetAttribute(void* pref, int, const void*, size_t) {
    return pref ? CUBLAS_STATUS_SUCCESS : CUBLAS_STATUS_INVALID_VALUE;
}

// One "algorithm": the library picks its tile configuration per call.
cublasStatus_t cublasLtMatmulAlgoGetHeuristic(void*, void*, void*, void*, void*, void*, void*,
                                              int requested, void* results, int* returned) {
    if (!results || !returned || requested < 1) return CUBLAS_STATUS_INVALID_VALUE;
    zlift_lt_heuristic_result* r = static_cast<zlift_lt_heuristic_result*>(results);
    std::memset(r, 0, sizeof *r);
    r->state = CUBLAS_STATUS_SUCCESS;
    r->wavesCount = 1.0f;
    *returned = 1;
    return CUBLAS_STATUS_SUCCESS;
}

cublasStatus_t cublasLtMatmul(void* lt, void* desc, const void* alpha, const void* A,
                              void* Adesc, const void* B, void* Bdesc, const void* beta,
                              const void* C, void* Cdesc, void* D, void* Ddesc, const void* algo,
                              void* workspace, size_t workspaceBytes, void* stream) {
    (void)algo; (void)workspace; (void)workspaceBytes;
    Handle* h = as_handle(lt);
    if (!h) return CUBLAS_STATUS_NOT_INITIALIZED;
    LtDesc* d = as_desc(desc);
    LtLayout *la = as_layout(Adesc), *lb = as_layout(Bdesc), *ld_ = as_layout(Ddesc);
    LtLayout* lc = Cdesc ? as_layout(Cdesc) : ld_;
    if (!d || !la || !lb || !ld_ || !lc) return CUBLAS_STATUS_INVALID_VALUE;
    if (la->order != CUBLASLT_ORDER_COL || lb->order != CUBLASLT_ORDER_COL ||
        lc->order != CUBLASLT_ORDER_COL || ld_->order != CUBLASLT_ORDER_COL)
        return CUBLAS_STATUS_NOT_SUPPORTED;
    const long long m = ld_->rows, n = ld_->cols;
    const long long k = d->transa == CUBLAS_OP_N ? la->cols : la->rows;
    const bool a_ok = d->transa == CUBLAS_OP_N ? la->rows == m : la->cols == m;
    const bool b_ok = d->transb == CUBLAS_OP_N ? (lb->rows == k && lb->cols == n)
                                               : (lb->rows == n && lb->cols == k);
    if (!a_ok || !b_ok || lc->rows != m || lc->cols != n) return CUBLAS_STATUS_INVALID_VALUE;
    if (m > 0x7fffffffLL || n > 0x7fffffffLL || k > 0x7fffffffLL)
        return CUBLAS_STATUS_NOT_SUPPORTED;
    const int batch = ld_->batch;
    if (la->batch != batch || lb->batch != batch || lc->batch != batch)
        return CUBLAS_STATUS_NOT_SUPPORTED;
    if (lc->type != ld_->type) return CUBLAS_STATUS_NOT_SUPPORTED;
    LtExtra x{};
    switch (d->epilogue) {
    case CUBLASLT_EPILOGUE_DEFAULT: x.epi = 0; break;
    case CUBLASLT_EPILOGUE_RELU: x.epi = kEpiRelu; break;
    case CUBLASLT_EPILOGUE_BIAS: x.epi = kEpiBias; break;
    case CUBLASLT_EPILOGUE_RELU_BIAS: x.epi = kEpiBias | kEpiRelu; break;
    case CUBLASLT_EPILOGUE_GELU: x.epi = kEpiGelu; break;
    case CUBLASLT_EPILOGUE_GELU_BIAS: x.epi = kEpiBias | kEpiGelu; break;
    default: return CUBLAS_STATUS_NOT_SUPPORTED;
    }
    if ((x.epi & kEpiBias) && !d->bias) return CUBLAS_STATUS_INVALID_VALUE;
    x.bias = d->bias;
    // bias in the output's 16-bit type, fp32 otherwise (zblas.c:696-704)
    x.bias_type = (ld_->type == kR16F || ld_->type == kR16BF) ? ld_->type : kR32F;
    x.stream = static_cast<cudaStream_t>(stream);
    x.pointer_mode = d->pointer_mode;
    x.scale_type = d->scale_type;
    // C != D: D starts as a copy of C (zblas.c:681-686), on the call's stream
    if (C && C != D && m > 0 && n > 0) {
        const size_t es = elem_size(ld_->type);
        for (int b = 0; b < batch; b++) {
            const char* src = static_cast<const char*>(C) + (size_t)b * lc->batch_stride * es;
            char* dst = static_cast<char*>(D) + (size_t)b * ld_->batch_stride * es;
            if (cudaMemcpy2DAsync(dst, ld_->ld * es, src, lc->ld * es, m * es, n,
                                  cudaMemcpyDeviceToDevice, x.stream) != cudaSuccess) {
                cudaGetLastError();
                return CUBLAS_STATUS_EXECUTION_FAILED;
            }
        }
    }
    const int compute = d->compute_type ? d->compute_type : kR32F;
    return gemm_ex(h, d->transa, d->transb, (int)m, (int)n, (int)k, alpha, A, la->type,
                   (int)la->ld, la->batch_stride, B, lb->type, (int)lb->ld, lb->batch_stride,
                   beta, D, ld_->type, (int)ld_->ld, ld_->batch_stride, batch, compute, &x);
}

#define ZLIFT_DEFINE_UNSUPPORTED(name)                       \
    cublasStatus_t name(void) {                              \
        trace("unsupported: %s", #name);                     \
        return CUBLAS_STATUS_NOT_SUPPORTED;                  \
    }
ZLIFT_UNSUPPORTED_LIST(ZLIFT_DEFINE_UNSUPPORTED)
#undef ZLIFT_DEFINE_UNSUPPORTED

int zlift_device_error(void) {
    cudaDeviceSynchronize();
    int e = gemm_tc_error(true);
    int e2 = gemm_simt_error(true);
    int e3 = fmha_error(true);
    int e4 = part_error(true);
    return e ? e : (e2 ? e2 : (e3 ? e3 : e4));
}

unsigned long long zlift_launch_count(void) { return launch_count(); }

int zlift_set_wait_limit_ns(unsigned long long ns) {
    if (ns == 0) return CUBLAS_STATUS_INVALID_VALUE;
    const int r = gemm_tc_set_wait_limit(ns) | gemm_simt_set_wait_limit(ns) |
                  fmha_set_wait_limit(ns) | part_set_wait_limit(ns);
    return r ? CUBLAS_STATUS_EXECUTION_FAILED : CUBLAS_STATUS_SUCCESS;
}

unsigned long long zlift_get_wait_limit_ns(void) { return wait_limit_ns(); }

int zlift_wait_probe(unsigned long long limit_ns, void* stream) {
    if (limit_ns == 0 || limit_ns > 10000000000ull) return CUBLAS_STATUS_INVALID_VALUE;
    return map_launch(wait_probe(limit_ns, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
