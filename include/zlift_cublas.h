/*
 * zlift_cublas.h -- the cuBLAS-style C ABI exported by libcublas.so.13.
 *
 * Drop-in for the reference's zblas shim (zLift, zblas/zblas.c), which a
 * CUDA program reaches by name through LD_PRELOAD / LD_LIBRARY_PATH
 * (zlift/src/run.rs:66-84).  Types are plain C: a status is an int, a
 * handle and a stream are opaque pointers, scalars are pointers whose
 * meaning follows the handle's pointer mode.
 *
 * Differences from the reference, all deliberate:
 *   - every GEMM runs on the GPU (sm_100a); there is no CPU fallback, so a
 *     case the GPU path cannot take returns a status instead;
 *   - calls are asynchronous on the handle's stream (the cuBLAS contract);
 *     the reference synchronises the whole context before every call
 *     (zblas/zblas.c:25-35) and waits after every kernel;
 *   - CUBLAS_POINTER_MODE_DEVICE is honoured (the reference stores the mode
 *     and always dereferences host pointers, zblas/zblas.c:77-79);
 *   - cublasGemmEx / cublasGemmStridedBatchedEx accept int8 inputs with an
 *     int32 output and CUBLAS_COMPUTE_32I (the reference returns
 *     NOT_SUPPORTED, zblas/zblas.c:366-367);
 *   - arguments are validated (negative sizes, short leading dimensions,
 *     null scalars) and answered with CUBLAS_STATUS_INVALID_VALUE.
 */
#ifndef ZLIFT_CUBLAS_H
#define ZLIFT_CUBLAS_H

#include <stddef.h>


#ifndef ZLIFT_API
#define ZLIFT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef int cublasStatus_t;          /* zblas/zblas.c:7 */
typedef void *cublasHandle_t;        /* zblas/zblas.c:8 */
typedef void *cudaStream_t_opaque;   /* zblas/zblas.c:9 (cudaStream_t) */

/* status codes: zblas/zblas.c:10-13, plus EXECUTION_FAILED (13) for a
 * kernel launch failure or a device-side wait that timed out */
#define CUBLAS_STATUS_SUCCESS 0
#define CUBLAS_STATUS_NOT_INITIALIZED 1
#define CUBLAS_STATUS_INVALID_VALUE 7
#define CUBLAS_STATUS_EXECUTION_FAILED 13
#define CUBLAS_STATUS_NOT_SUPPORTED 15

/* enums: zblas/zblas.c:14-15, :305 */
#define CUBLAS_OP_N 0
#define CUBLAS_OP_T 1
#define CUBLAS_OP_C 2
#define CUBLAS_DEFAULT_MATH 0
#define CUBLAS_TF32_TENSOR_OP_MATH 3
#define CUBLAS_POINTER_MODE_HOST 0
#define CUBLAS_POINTER_MODE_DEVICE 1
#define CUDA_R_32F 0
#define CUDA_R_16F 2
#define CUDA_R_8I 3
#define CUDA_R_32I 10
#define CUDA_R_16BF 14
#define CUBLAS_COMPUTE_32F 68
#define CUBLAS_COMPUTE_32I 72

/* ---- handle, stream and mode (zblas/zblas.c:42-76, :454-470) ---------- */
ZLIFT_API cublasStatus_t cublasCreate_v2(cublasHandle_t *handle);               /* zblas.c:42 */
ZLIFT_API cublasStatus_t cublasDestroy_v2(cublasHandle_t handle);               /* zblas.c:50 */
ZLIFT_API cublasStatus_t cublasGetVersion_v2(cublasHandle_t handle, int *ver);  /* zblas.c:51 */
ZLIFT_API cublasStatus_t cublasSetStream_v2(cublasHandle_t handle, void *stream);   /* zblas.c:57 */
ZLIFT_API cublasStatus_t cublasGetStream_v2(cublasHandle_t handle, void **stream);  /* zblas.c:62 */
ZLIFT_API cublasStatus_t cublasSetPointerMode_v2(cublasHandle_t handle, int mode);  /* zblas.c:67 */
ZLIFT_API cublasStatus_t cublasGetPointerMode_v2(cublasHandle_t handle, int *mode); /* zblas.c:72 */
ZLIFT_API cublasStatus_t cublasSetMathMode(cublasHandle_t handle, int mode);        /* zblas.c:460 */
ZLIFT_API cublasStatus_t cublasGetMathMode(cublasHandle_t handle, int *mode);       /* zblas.c:465 */
ZLIFT_API cublasStatus_t cublasSetWorkspace_v2(cublasHandle_t handle, void *workspace,
                                     size_t bytes);                      /* zblas.c:454 */
ZLIFT_API cublasStatus_t cublasSetSmCountTarget(cublasHandle_t handle, int count);  /* zblas.c:471 */
ZLIFT_API cublasStatus_t cublasGetSmCountTarget(cublasHandle_t handle, int *count); /* zblas.c:475 */
ZLIFT_API const char *cublasGetStatusName(cublasStatus_t status);         /* zblas.c:232 */
ZLIFT_API const char *cublasGetStatusString(cublasStatus_t status);       /* cuBLAS API */

/* ---- GEMM entry points ------------------------------------------------ */

/* fp32 GEMM, column-major: C = alpha*op(A)*op(B) + beta*C.
 * Replaces zblas/zblas.c:111-130 (XMX 3-pass bf16 split or cblas_sgemm).
 * Default math: 3-product tf32 split on the tensor cores (fp32-accurate);
 * CUBLAS_TF32_TENSOR_OP_MATH: one tf32 product. */
ZLIFT_API cublasStatus_t cublasSgemm_v2(cublasHandle_t handle, int transa, int transb,
                              int m, int n, int k, const float *alpha,
                              const float *A, int lda, const float *B, int ldb,
                              const float *beta, float *C, int ldc);

/* fp64 GEMM.  zblas/zblas.c:131-144 (cublasDgemm_v2: oneMKL on the GPU,
 * zblas_gpu.cpp:1548-1559, else cblas_dgemm on the host).  Here: a CUDA-core
 * fp64 kernel (B200's tensor cores have no fp64 form in tcgen05); alpha and
 * beta are double, host or device pointer mode. */
ZLIFT_API cublasStatus_t cublasDgemm_v2(cublasHandle_t handle, int transa, int transb, int m,
                                        int n, int k, const double *alpha, const double *A,
                                        int lda, const double *B, int ldb, const double *beta,
                                        double *C, int ldc);

/* Mixed-type GEMM.  Replaces zblas/zblas.c:357-391.
 *   A,B fp16  -> C fp16 or fp32, compute 32F (0 or 68)
 *   A,B bf16  -> C bf16 or fp32, compute 32F
 *   A,B,C fp32, compute 32F     -> cublasSgemm_v2
 *   A,B int8  -> C int32, compute 32I (72, or legacy CUDA_R_32I = 10);
 *               alpha/beta are int32_t.  New: not in the reference.
 * `algo` is ignored, as in the reference (zblas.c:364). */
ZLIFT_API cublasStatus_t cublasGemmEx(cublasHandle_t handle, int transa, int transb,
                            int m, int n, int k, const void *alpha,
                            const void *A, int Atype, int lda,
                            const void *B, int Btype, int ldb,
                            const void *beta, void *C, int Ctype, int ldc,
                            int computeType, int algo);

/* Batched form with element strides; one launch for the whole batch.
 * Replaces zblas/zblas.c:491-511 (a host loop of cublasGemmEx calls). */
ZLIFT_API cublasStatus_t cublasGemmStridedBatchedEx(
    cublasHandle_t handle, int transa, int transb, int m, int n, int k,
    const void *alpha, const void *A, int Atype, int lda, long long strideA,
    const void *B, int Btype, int ldb, long long strideB, const void *beta,
    void *C, int Ctype, int ldc, long long strideC, int batchCount,
    int computeType, int algo);

/* fp32 strided-batched GEMM.  Replaces zblas/zblas.c:145-168. */
ZLIFT_API cublasStatus_t cublasSgemmStridedBatched(
    cublasHandle_t handle, int transa, int transb, int m, int n, int k,
    const float *alpha, const float *A, int lda, long long strideA,
    const float *B, int ldb, long long strideB, const float *beta, float *C,
    int ldc, long long strideC, int batchCount);

/* cublasGemmEx with 32F compute and float scalars.  zblas/zblas.c:480-487. */
ZLIFT_API cublasStatus_t cublasSgemmEx(cublasHandle_t handle, int transa, int transb,
                             int m, int n, int k, const float *alpha,
                             const void *A, int Atype, int lda,
                             const void *B, int Btype, int ldb,
                             const float *beta, void *C, int Ctype, int ldc);

/* fp16 GEMM with fp16 scalars (bit patterns).  zblas/zblas.c:278-304.
 * Accumulates in fp32, like the reference's host path. */
ZLIFT_API cublasStatus_t cublasHgemm(cublasHandle_t handle, int transa, int transb,
                           int m, int n, int k, const unsigned short *alpha,
                           const unsigned short *A, int lda,
                           const unsigned short *B, int ldb,
                           const unsigned short *beta, unsigned short *C,
                           int ldc);

/* fp32 GEMM with the arguments and results of cublasSgemm_v2 that
 * allocates no device memory.  No counterpart in the reference.
 * For callers that must not call cudaMalloc: code inside a CUDA-graph
 * capture that may not allocate, programs whose device memory is already
 * fully reserved, and interposition layers (like zLift's, which answers a
 * program's cuBLAS calls from inside that program) that must leave the
 * program's allocations alone.  cublasSgemm_v2 keeps its tf32 split planes
 * in scratch it allocates per handle; this entry keeps them in a fixed
 * 16 MiB array of the library's device image (per GPU, held until exit).
 * Limit: 4 * P * (m*kp + n*kp) bytes <= 16 MiB, kp = k rounded up to 4,
 * P = 2 (default math) or 1 (CUBLAS_TF32_TENSOR_OP_MATH); larger calls
 * return CUBLAS_STATUS_INVALID_VALUE.  The first call on a device looks up
 * the array's address there -- make it before any stream capture.  All
 * calls share the array: calls whose kernels overlap on the GPU race, so
 * keep them on one stream. */
ZLIFT_API cublasStatus_t zlift_sgemm_noalloc(cublasHandle_t handle, int transa, int transb,
                                             int m, int n, int k, const float *alpha,
                                             const float *A, int lda, const float *B, int ldb,
                                             const float *beta, float *C, int ldc);

/* ---- library extras (no reference counterpart) ------------------------ */

/* Returns and clears the device error word: 0 if no kernel of this library
 * has recorded an error on the current device since the last call,
 * otherwise 1 (a bounded device-side wait timed out).  Synchronises the
 * current device. */
ZLIFT_API int zlift_device_error(void);

/* Number of kernels this library launched on any stream since load. */
ZLIFT_API unsigned long long zlift_launch_count(void);

/* Time limit, in nanoseconds, of every bounded device-side wait of this
 * library's kernels on the current device (default 2 s).  A wait that runs
 * out records error 1 (see zlift_device_error), makes its kernel leave its
 * loops and return; the context stays usable.  ns = 0 is INVALID_VALUE. */
ZLIFT_API int zlift_set_wait_limit_ns(unsigned long long ns);
ZLIFT_API unsigned long long zlift_get_wait_limit_ns(void);

/* Failure-path check: launches on `stream` a one-thread kernel whose
 * mbarrier wait nothing completes, bounded by limit_ns (at most 10 s).  It
 * returns after the limit with error 1 recorded for zlift_device_error.
 * The reference's failure handling is decline-then-fallback
 * (zblas/zblas_gpu.cpp:184-201); this exercises the build's replacement,
 * the bounded wait, without faulting or hanging the GPU. */
ZLIFT_API int zlift_wait_probe(unsigned long long limit_ns, void *stream);

#ifdef __cplusplus
}
#endif
#endif
