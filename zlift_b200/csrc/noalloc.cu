// noalloc.cu -- zlift_sgemm_noalloc: the fp32 GEMM of cublasSgemm_v2 for
// callers that cannot allocate device memory.
//
// Who needs it: code that runs where cudaMalloc is off limits -- inside a
// CUDA-graph capture that must not allocate, under a memory pool that is
// already fully reserved, or in an interposition layer (such as zLift's,
// which answers a program's cuBLAS calls from inside that program) that
// must not change the program's allocation pattern.  cublasSgemm_v2 keeps
// its tf32 split planes in per-handle scratch it allocates on first use;
// this entry point keeps them in a fixed array in the library's device
// image instead, so no call allocates anything.
//
// The array: kScratchBytes (16 MiB) of device memory per GPU that loads the
// library, held until the process exits.  A call needs
//   4 bytes * P * (m*kp + n*kp),  kp = k rounded up to a multiple of 4,
// with P = 2 planes per operand under the default math mode (hi and lo)
// and P = 1 under CUBLAS_TF32_TENSOR_OP_MATH, each operand's planes
// rounded up to 256 bytes; larger calls are rejected with
// CUBLAS_STATUS_INVALID_VALUE.  (1024^3 with the default math needs
// 16 MiB exactly.)
//
// The first call on a device looks up that device's address of the array
// (cudaGetSymbolAddress, with the device current) and caches it, tagged
// with the current context (a new context -- after cudaDeviceReset, say --
// looks it up again); make that first call before any stream capture
// begins.  Every call on a device
// shares the one array and overwrites all of the planes it reads, so no
// call depends on what an earlier call left there -- but two calls whose
// kernels overlap on the GPU (different streams, or different host
// threads) race on the array: order them on one stream.
#include "gemm.h"

#include "../../include/zlift_cublas.h"

#include <cuda.h>

#include <cstdio>
#include <mutex>

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;

static __device__ __align__(256) float g_noalloc_scratch[kScratchBytes / sizeof(float)];

std::mutex g_mu;

// The driver's cuCtxGetCurrent, looked up once (the library links only the
// runtime).
using CtxGetCurrentFn = CUresult (*)(CUcontext*);
CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) ==
                cudaSuccess && q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<CtxGetCurrentFn>(f);
        else
            cudaGetLastError();
    });
    return fn;
}

// One cached address per device, tagged with the context it was looked up
// in: after cudaDeviceReset, or under another context on the same device,
// the array lives at a new address and is looked up again.
struct Cached {
    CUcontext ctx = nullptr;
    void* addr = nullptr;
};
Cached g_addr[64];

// Device address of g_noalloc_scratch in the current context.  Host code
// may not use the array's name as an address.
float* scratch_on_current_device() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return nullptr;
    }
    CUcontext ctx = nullptr;
    CtxGetCurrentFn get = ctx_get_current();
    if (get && get(&ctx) == CUDA_SUCCESS && !ctx) {
        // no context yet on this thread: the symbol lookup creates the
        // device's primary context as a side effect
        void* p = nullptr;
        cudaGetSymbolAddress(&p, g_noalloc_scratch);
        cudaGetLastError();
        get(&ctx);
    }
    if (!get || !ctx) {
        fprintf(stderr, "[zblas] zlift_sgemm_noalloc: no current CUDA context\n");
        return nullptr;
    }
    std::lock_guard<std::mutex> lock(g_mu);
    Cached& c = g_addr[dev];
    if (!c.addr || c.ctx != ctx) {
        void* p = nullptr;
        cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            cudaGetLastError();
            fprintf(stderr, "[zblas] zlift_sgemm_noalloc: cudaGetSymbolAddress failed: %s\n",
                    cudaGetErrorString(e));
            return nullptr;
        }
        c.ctx = ctx;
        c.addr = p;
    }
    return static_cast<float*>(c.addr);
}

cublasStatus_t done(int rc) {
    if (rc == 0) return CUBLAS_STATUS_SUCCESS;
    cudaGetLastError();
    return CUBLAS_STATUS_EXECUTION_FAILED;
}

}  // namespace

extern "C" cublasStatus_t zlift_sgemm_noalloc(cublasHandle_t handle, int transa, int transb,
                                              int m, int n, int k, const float* alpha,
                                              const float* A, int lda, const float* B, int ldb,
                                              const float* beta, float* C, int ldc) {
    using namespace zl;
    if (!handle) return CUBLAS_STATUS_NOT_INITIALIZED;
    void* sv = nullptr;
    int pmode = 0, mmode = 0;
    if (cublasGetStream_v2(handle, &sv) || cublasGetPointerMode_v2(handle, &pmode) ||
        cublasGetMathMode(handle, &mmode))
        return CUBLAS_STATUS_NOT_INITIALIZED;
    cudaStream_t s = static_cast<cudaStream_t>(sv);
    if (transa < 0 || transa > 2 || transb < 0 || transb > 2 || m < 0 || n < 0 || k < 0)
        return CUBLAS_STATUS_INVALID_VALUE;
    const int ra = transa == CUBLAS_OP_N ? m : k, rb = transb == CUBLAS_OP_N ? k : n;
    if (lda < (ra > 1 ? ra : 1) || ldb < (rb > 1 ? rb : 1) || ldc < (m > 1 ? m : 1))
        return CUBLAS_STATUS_INVALID_VALUE;
    if (m == 0 || n == 0) return CUBLAS_STATUS_SUCCESS;
    if (!alpha || !beta || !C || (k > 0 && (!A || !B))) return CUBLAS_STATUS_INVALID_VALUE;

    GemmDesc d{};
    d.transa = transa == CUBLAS_OP_N ? 0 : 1;
    d.transb = transb == CUBLAS_OP_N ? 0 : 1;
    d.m = m; d.n = n; d.k = k; d.batch = 1;
    d.A = A; d.lda = lda; d.Atype = kR32F;
    d.B = B; d.ldb = ldb; d.Btype = kR32F;
    d.C = C; d.ldc = ldc; d.Ctype = kR32F;
    d.kind = mmode == CUBLAS_TF32_TENSOR_OP_MATH ? Kind::TF32 : Kind::TF32X3;
    if (pmode == CUBLAS_POINTER_MODE_DEVICE) {
        d.alpha_dev = alpha;
        d.beta_dev = beta;
    } else {
        d.alpha = *alpha;
        d.beta = *beta;
    }
    if (k == 0) return done(gemm_simt(d, s));   // C = beta * C, no planes

    const bool two = d.kind == Kind::TF32X3;
    const long long kp = ((long long)k + 3) & ~3ll;
    auto up = [](long long e) { return (e + 63) & ~63ll; };
    // Size check without overflow: every factor is bounded before the
    // products are formed (m, n < 2^31 and kp < 2^31 + 4, so m*kp < 2^63;
    // each plane is then compared with the array before they are summed).
    const unsigned long long cap = kScratchBytes / sizeof(float);     // floats in the array
    const unsigned long long ea_u = (unsigned long long)m * (unsigned long long)kp;
    const unsigned long long eb_u = (unsigned long long)n * (unsigned long long)kp;
    const unsigned long long planes = two ? 2 : 1;
    bool fits = ea_u <= cap && eb_u <= cap;
    long long ea = 0, eb = 0;
    unsigned long long need = ~0ull;
    if (fits) {
        ea = up((long long)ea_u);
        eb = up((long long)eb_u);
        need = planes * ((unsigned long long)ea + (unsigned long long)eb) * sizeof(float);
        fits = need <= kScratchBytes;
    }
    if (!fits) {
        fprintf(stderr,
                "[zblas] zlift_sgemm_noalloc: %dx%dx%d needs more scratch than the fixed "
                "array's %zu bytes\n", m, n, k, kScratchBytes);
        return CUBLAS_STATUS_INVALID_VALUE;
    }
    float* base = scratch_on_current_device();
    if (!base) return CUBLAS_STATUS_EXECUTION_FAILED;
    float* a_hi = base;
    float* b_hi = a_hi + ea;
    float* a_lo = two ? b_hi + eb : nullptr;
    float* b_lo = two ? a_lo + ea : nullptr;
    int rc = split_tf32(A, d.transa != 0, m, k, lda, 0, 1, kp, a_hi, a_lo, s);
    if (rc == 0) rc = split_tf32(B, d.transb == 0, n, k, ldb, 0, 1, kp, b_hi, b_lo, s);
    if (rc) return done(rc);
    GemmDesc e = d;
    e.transa = 1;
    e.transb = 0;
    e.A = a_hi; e.B = b_hi;
    e.lda = kp; e.ldb = kp;
    e.strideA = (long long)m * kp;
    e.strideB = (long long)n * kp;
    e.A_hi = a_hi; e.A_lo = a_lo; e.B_hi = b_hi; e.B_lo = b_lo;
    rc = gemm_tc(e, s);
    if (rc == 1) rc = gemm_simt(d, s);   // plain fp32 on CUDA cores, no planes
    return done(rc);
}
