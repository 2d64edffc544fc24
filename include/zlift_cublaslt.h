/*
 * zlift_cublaslt.h -- the cuBLASLt subset and the unsupported-entry stubs
 * exported by libcublas.so.13, as the reference's zblas exports them
 * (zblas/zblas.c:512-734).
 *
 * cublasLtMatmul runs as one GEMM launch with the epilogue (bias per row,
 * ReLU, GELU in its tanh form) fused into the GEMM's epilogue, on the stream
 * passed to the call.  The reference runs the GEMM and then a separate
 * epilogue pass (GPU zblas_gpu.cpp:1040-1089 or host zblas.c:674-710).
 * Attribute and enum numbers are cuBLASLt's (the reference uses the same).
 */
#ifndef ZLIFT_CUBLASLT_H
#define ZLIFT_CUBLASLT_H

#include <stddef.h>

#include "zlift_cublas.h"

#ifndef ZLIFT_API
#define ZLIFT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef void *cublasLtHandle_t;

/* matmul descriptor attributes (zblas.c:512-516) */
#define CUBLASLT_MATMUL_DESC_COMPUTE_TYPE 0
#define CUBLASLT_MATMUL_DESC_SCALE_TYPE 1
#define CUBLASLT_MATMUL_DESC_POINTER_MODE 2
#define CUBLASLT_MATMUL_DESC_TRANSA 3
#define CUBLASLT_MATMUL_DESC_TRANSB 4
#define CUBLASLT_MATMUL_DESC_TRANSC 5
#define CUBLASLT_MATMUL_DESC_FILL_MODE 6
#define CUBLASLT_MATMUL_DESC_EPILOGUE 7
#define CUBLASLT_MATMUL_DESC_BIAS_POINTER 8
/* matrix layout attributes (zblas.c:517-521) */
#define CUBLASLT_MATRIX_LAYOUT_TYPE 0
#define CUBLASLT_MATRIX_LAYOUT_ORDER 1
#define CUBLASLT_MATRIX_LAYOUT_ROWS 2
#define CUBLASLT_MATRIX_LAYOUT_COLS 3
#define CUBLASLT_MATRIX_LAYOUT_LD 4
#define CUBLASLT_MATRIX_LAYOUT_BATCH_COUNT 5
#define CUBLASLT_MATRIX_LAYOUT_STRIDED_BATCH_OFFSET 6
#define CUBLASLT_ORDER_COL 0
/* epilogues (zblas.c:522-525) */
#define CUBLASLT_EPILOGUE_DEFAULT 1
#define CUBLASLT_EPILOGUE_RELU 2
#define CUBLASLT_EPILOGUE_BIAS 4
#define CUBLASLT_EPILOGUE_RELU_BIAS 6
#define CUBLASLT_EPILOGUE_GELU 32
#define CUBLASLT_EPILOGUE_GELU_BIAS 36

/* heuristic result, laid out as cuBLASLt's (zblas.c:620-625) */
typedef struct {
    unsigned long long algo[8];
    size_t workspaceSize;
    cublasStatus_t state;
    float wavesCount;
    int reserved[4];
} zlift_lt_heuristic_result;

/* Lt handles are this library's cuBLAS handles; a handle from
 * cublasCreate_v2 is accepted too (the reference passes its Lt handle to
 * cublasGemmEx, zblas.c:687-691). */
ZLIFT_API cublasStatus_t cublasLtCreate(cublasLtHandle_t *handle);
ZLIFT_API cublasStatus_t cublasLtDestroy(cublasLtHandle_t handle);
ZLIFT_API cublasStatus_t cublasLtGetVersion(void);                            /* zblas.c:538 */
ZLIFT_API cublasStatus_t cublasLtMatmulDescCreate(void **desc, int computeType,
                                                  int scaleType);              /* zblas.c:539 */
ZLIFT_API cublasStatus_t cublasLtMatmulDescDestroy(void *desc);               /* zblas.c:549 */
ZLIFT_API cublasStatus_t cublasLtMatmulDescSetAttribute(void *desc, int attr, const void *buf,
                                                        size_t bytes);         /* zblas.c:550 */
ZLIFT_API cublasStatus_t cublasLtMatmulDescGetAttribute(void *desc, int attr, void *buf,
                                                        size_t bytes, size_t *written); /* :566 */
ZLIFT_API cublasStatus_t cublasLtMatrixLayoutCreate(void **layout, int type,
                                                    unsigned long long rows,
                                                    unsigned long long cols,
                                                    long long ld);             /* zblas.c:578 */
ZLIFT_API cublasStatus_t cublasLtMatrixLayoutDestroy(void *layout);           /* zblas.c:589 */
ZLIFT_API cublasStatus_t cublasLtMatrixLayoutSetAttribute(void *layout, int attr,
                                                          const void *buf, size_t bytes); /* :590 */
ZLIFT_API cublasStatus_t cublasLtMatmulPreferenceCreate(void **pref);         /* zblas.c:606 */
ZLIFT_API cublasStatus_t cublasLtMatmulPreferenceDestroy(void *pref);         /* zblas.c:613 */
ZLIFT_API cublasStatus_t cublasLtMatmulPreferenceSetAttribute(void *pref, int attr,
                                                              const void *buf, size_t bytes);
ZLIFT_API cublasStatus_t cublasLtMatmulAlgoGetHeuristic(void *lt, void *desc, void *Adesc,
                                                        void *Bdesc, void *Cdesc, void *Ddesc,
                                                        void *pref, int requested,
                                                        void *results, int *returned); /* :626 */
/* D = epilogue(alpha * op(A) * op(B) + beta * C), column-major layouts,
 * batched when the layouts carry a batch count.  zblas.c:643-711.
 * New (the reference has no int8 path): int8 A/B with compute 32I give an
 * int32 D (int32 scalars, scale type CUDA_R_32I), or, with int8 C/D and
 * scale type CUDA_R_32F, the requantised int8 D = saturate(round(alpha *
 * acc + beta * C)) (float scalars, round to nearest even, [-128, 127]);
 * int8 outputs take no bias/activation epilogue (NOT_SUPPORTED). */
ZLIFT_API cublasStatus_t cublasLtMatmul(void *lt, void *desc, const void *alpha,
                                        const void *A, void *Adesc, const void *B, void *Bdesc,
                                        const void *beta, const void *C, void *Cdesc, void *D,
                                        void *Ddesc, const void *algo, void *workspace,
                                        size_t workspaceBytes, void *stream);

/* Entry points the reference exports as NOT_SUPPORTED (zblas.c:712-734);
 * exported here the same way so programs linked against them still load.
 * Each returns CUBLAS_STATUS_NOT_SUPPORTED. */
#define ZLIFT_UNSUPPORTED_LIST(X) \
    X(cublasCdotc_v2) X(cublasCdotu_v2) X(cublasZdotc_v2) X(cublasZdotu_v2) X(cublasDotEx) \
    X(cublasCgemm_v2) X(cublasZgemm_v2) X(cublasCgemv_v2) X(cublasZgemv_v2) \
    X(cublasCgemmStridedBatched) X(cublasZgemmStridedBatched) X(cublasDgemmStridedBatched) \
    X(cublasStrsm_v2) X(cublasDtrsm_v2) X(cublasCtrsm_v2) X(cublasZtrsm_v2) \
    X(cublasStrsmBatched) X(cublasDtrsmBatched) X(cublasCtrsmBatched) X(cublasZtrsmBatched) \
    X(cublasSgetrfBatched) X(cublasDgetrfBatched) X(cublasCgetrfBatched) X(cublasZgetrfBatched) \
    X(cublasSgetrsBatched) X(cublasDgetrsBatched) X(cublasCgetrsBatched) X(cublasZgetrsBatched) \
    X(cublasSgeqrfBatched) X(cublasDgeqrfBatched) X(cublasCgeqrfBatched) X(cublasZgeqrfBatched) \
    X(cublasSgelsBatched) X(cublasDgelsBatched) X(cublasCgelsBatched) X(cublasZgelsBatched)

#define ZLIFT_DECLARE_UNSUPPORTED(name) ZLIFT_API cublasStatus_t name(void);
ZLIFT_UNSUPPORTED_LIST(ZLIFT_DECLARE_UNSUPPORTED)
#undef ZLIFT_DECLARE_UNSUPPORTED

#ifdef __cplusplus
}
#endif
#endif
