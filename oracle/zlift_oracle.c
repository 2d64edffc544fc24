/*
 * zlift_oracle.c -- TEST INFRASTRUCTURE, NOT PRODUCT CODE.
 *
 * A plain-C restatement of the reference's CPU arithmetic for the GEMM and
 * fused-attention hot path.  It is the checker for the CUDA kernels in
 * zlift_b200/csrc: only tests/, __graft_entry__.smoke() and bench.py's CPU
 * baseline leg may load it.  The product library never links or calls it.
 *
 * What each function restates (paths relative to the zLift project root):
 *   zo_half_to_float / zo_float_to_half  zblas/zblas.c:241-277
 *       (fp16 RNE for normals, TRUNCATION for subnormals, overflow -> inf)
 *   zo_bf16_to_float / zo_float_to_bf16  zblas/zblas.c:306-317
 *       (bf16 RNE with no NaN special case)
 *   zo_sgemm                              cblas_sgemm as called at
 *       zblas/zblas.c:127 (column-major, op in {N,T,C}); products are summed
 *       in double and rounded once, which is at least as accurate as the
 *       single-precision BLAS the reference links.
 *   zo_gemm_ex                            cublasGemmEx, zblas/zblas.c:357-391,
 *       with gemm_ex_host (zblas/zblas.c:318-356): widen A/B (and a narrow C)
 *       to fp32, run the fp32 GEMM, narrow C with the reference converter.
 *       The int8 x int8 -> int32 branch (Atype=Btype=CUDA_R_8I, Ctype=
 *       CUDA_R_32I, compute 32I) has no counterpart in the reference (which
 *       returns NOT_SUPPORTED, zblas/zblas.c:366-367); it is exact int32
 *       arithmetic with two's-complement wrap for alpha/beta scaling.
 *   zo_gemm_i8_s8                         cublasLtMatmul's int8-output form
 *       (int8 A/B/C/D, compute 32I, scale type 32F; not in the reference):
 *       the exact int32 product, x = alpha * float(acc) (+ fmaf(beta,
 *       float(C), x)), rounded to nearest even and saturated to int8.
 *   zo_dgemm                              cblas_dgemm as called at
 *       zblas/zblas.c:131-144 (fp64, summed in K order).
 *   zo_gemm_strided_batched_ex            zblas/zblas.c:491-511 (host loop
 *       over the batch; strides in elements, elem_size :488-490).
 *   zo_lt_epilogue                        cublasLtMatmul's bias / ReLU /
 *       GELU pass, zblas/zblas.c:692-710 with gelu_tanh :638-642.
 *   zo_attention / zo_attention_rows      the fp32 math of fmha_f32
 *       (zblas/zblas_gpu.cpp:793-844) with the masking and rounding points
 *       of fmha_run (zblas/zblas_gpu.cpp:892-1039): an optional additive
 *       bias after the scaling (:963-966, :822-823), causal mask
 *       `key > query + diag` (:967), fully-masked rows give O = 0 (:981,
 *       :991, :1015), P rounded to the input type before P.V (:1001, via
 *       joint_matrix_copy), O accumulated wide and rounded once (:1013-1023).
 *       The log-sum-exp output (natural log, m + log(l)) is not produced by
 *       the reference at all; it follows the flash-attention convention.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

enum { ZO_OP_N = 0, ZO_OP_T = 1, ZO_OP_C = 2 };
enum { ZO_R_32F = 0, ZO_R_16F = 2, ZO_R_8I = 3, ZO_R_32I = 10, ZO_R_16BF = 14 };
enum { ZO_COMPUTE_32F = 68, ZO_COMPUTE_32I = 72 };
enum { ZO_OK = 0, ZO_NOT_INITIALIZED = 1, ZO_INVALID_VALUE = 7,
       ZO_NOT_SUPPORTED = 15 };

/* ---- scalar converters (zblas/zblas.c:241-277, :306-317) -------------- */

float zo_half_to_float(uint16_t h) {
    uint32_t sign = (h >> 15) & 1u, ex = (h >> 10) & 0x1fu, man = h & 0x3ffu;
    uint32_t bits;
    if (ex == 0) {
        if (man == 0) {
            bits = sign << 31;
        } else {                       /* subnormal: renormalise */
            int shift = 0;
            while (!(man & 0x400u)) { man <<= 1; shift++; }
            /* value = 1.m * 2^(-14 - (shift - 1)) ... written via exponent */
            bits = (sign << 31) | ((uint32_t)(127 - 15 - (shift - 1)) << 23)
                 | ((man & 0x3ffu) << 13);
        }
    } else if (ex == 31) {
        bits = (sign << 31) | 0x7f800000u | (man << 13);
    } else {
        bits = (sign << 31) | ((ex - 15u + 127u) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

uint16_t zo_float_to_half(float f) {
    uint32_t bits;
    memcpy(&bits, &f, 4);
    uint32_t sign = (bits >> 16) & 0x8000u;
    int ex = (int)((bits >> 23) & 0xffu) - 127;
    uint32_t man = bits & 0x7fffffu;
    if (ex > 15) return (uint16_t)(sign | 0x7c00u);      /* overflow, inf, NaN */
    if (ex < -24) return (uint16_t)sign;                 /* underflow to zero */
    if (ex < -14) {                                      /* subnormal: truncate */
        man |= 0x800000u;
        return (uint16_t)(sign | (man >> (13 + (-14 - ex))));
    }
    uint32_t h = sign | ((uint32_t)(ex + 15) << 10) | (man >> 13);
    uint32_t rem = man & 0x1fffu;                        /* round to nearest even */
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)h;
}

float zo_bf16_to_float(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    memcpy(&f, &u, 4);
    return f;
}

uint16_t zo_float_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

/* bulk forms, used by the tests to pin the converters element by element */
void zo_half_to_float_n(const uint16_t *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = zo_half_to_float(x[i]);
}
void zo_float_to_half_n(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = zo_float_to_half(x[i]);
}
void zo_bf16_to_float_n(const uint16_t *x, float *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = zo_bf16_to_float(x[i]);
}
void zo_float_to_bf16_n(const float *x, uint16_t *y, int64_t n) {
    for (int64_t i = 0; i < n; i++) y[i] = zo_float_to_bf16(x[i]);
}

/* ---- column-major operand access ------------------------------------ */

/* element (i, l) of op(X), where X is stored column-major with leading
 * dimension ld: op N reads X[i + l*ld], op T/C reads X[l + i*ld]. */
static inline int64_t opidx(int op, int64_t i, int64_t l, int64_t ld) {
    return op == ZO_OP_N ? i + l * ld : l + i * ld;
}

static double load_elem(const void *p, int type, int64_t at) {
    switch (type) {
    case ZO_R_32F: return ((const float *)p)[at];
    case ZO_R_16F: return zo_half_to_float(((const uint16_t *)p)[at]);
    case ZO_R_16BF: return zo_bf16_to_float(((const uint16_t *)p)[at]);
    case ZO_R_8I: return ((const int8_t *)p)[at];
    case ZO_R_32I: return ((const int32_t *)p)[at];
    default: return 0.0;
    }
}

static int gemm_wide(int transa, int transb, int m, int n, int k, float alpha,
                     const void *A, int Atype, int lda, const void *B, int Btype,
                     int ldb, float beta, void *C, int Ctype, int ldc);

/* fp32 GEMM restating cblas_sgemm (zblas/zblas.c:127): C = alpha*op(A)op(B)
 * + beta*C, column-major.  beta == 0 does not read C (BLAS convention).
 * Products are summed in fp64 and rounded once (gemm_wide); the plain loop
 * below only runs if the packed copies cannot be allocated. */
void zo_sgemm(int transa, int transb, int m, int n, int k, float alpha,
              const float *A, int lda, const float *B, int ldb, float beta,
              float *C, int ldc) {
    if (gemm_wide(transa, transb, m, n, k, alpha, A, ZO_R_32F, lda, B, ZO_R_32F, ldb,
                  beta, C, ZO_R_32F, ldc) == ZO_OK)
        return;
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        for (int i = 0; i < m; i++) {
            double acc = 0.0;
            for (int l = 0; l < k; l++)
                acc += (double)A[opidx(transa, i, l, lda)]
                     * (double)B[opidx(transb, l, j, ldb)];
            double c = (double)alpha * acc;
            if (beta != 0.0f) c += (double)beta * (double)C[i + (int64_t)j * ldc];
            C[i + (int64_t)j * ldc] = (float)c;
        }
    }
}

/* Dot product of two int8 vectors with int32 wrap-around accumulation.
 * Accumulating in 32 bits modulo 2^32 gives the same low 32 bits as an
 * exact (wider) sum, which is all the int32 result keeps.  Written so the
 * compiler vectorises it; the clones pick AVX2 / AVX-512 where the host
 * has them. */
__attribute__((target_clones("arch=skylake-avx512", "avx2", "default")))
static uint32_t dot_i8(const int8_t *a, const int8_t *b, int k) {
    uint32_t acc = 0;
    for (int l = 0; l < k; l++)
        acc += (uint32_t)((int32_t)a[l] * (int32_t)b[l]);
    return acc;
}

/* op(X) as a dense [rows][k] int8 array (K contiguous). */
static int8_t *pack_i8(int op, const int8_t *X, int rows, int k, int ld, int is_b) {
    int8_t *p = malloc((size_t)rows * (size_t)(k > 0 ? k : 1));
    if (!p) return NULL;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int l = 0; l < k; l++)
            /* A: op(A)(r, l); B: op(B)(l, r) */
            p[(size_t)r * k + l] = is_b ? X[opidx(op, l, r, ld)] : X[opidx(op, r, l, ld)];
    return p;
}

/* fp64 GEMM restating cblas_dgemm (zblas/zblas.c:131-144): products summed
 * in fp64 in K order, C = alpha*sum + beta*C (beta == 0 does not read C). */
void zo_dgemm(int transa, int transb, int m, int n, int k, double alpha,
              const double *A, int lda, const double *B, int ldb, double beta,
              double *C, int ldc) {
#pragma omp parallel for schedule(static)
    for (int j = 0; j < n; j++) {
        for (int i = 0; i < m; i++) {
            double acc = 0.0;
            for (int l = 0; l < k; l++)
                acc += A[opidx(transa, i, l, lda)] * B[opidx(transb, l, j, ldb)];
            double c = alpha * acc;
            if (beta != 0.0) c += beta * C[i + (int64_t)j * ldc];
            C[i + (int64_t)j * ldc] = c;
        }
    }
}

/* int8 output with float scaling (cuBLASLt's int8 D with scale type 32F):
 * x = alpha * float(acc), plus fmaf(beta, float(C), x) when beta != 0, then
 * rounded to nearest with ties to even (lrintf in the default rounding
 * mode) and saturated to [-128, 127]; NaN gives 0. */
static int8_t requant_s8(int32_t acc, float alpha, float beta, int8_t old) {
    float x = alpha * (float)acc;
    if (beta != 0.0f) x = fmaf(beta, (float)old, x);
    if (x != x) return 0;
    if (x >= 127.0f) return 127;
    if (x <= -128.0f) return -128;
    return (int8_t)lrintf(x);
}

/* int8 x int8 products, exact with int32 wrap-around.  C8 == NULL: int32
 * C = alpha * acc + beta * C with int32 alpha/beta (wrapping); otherwise
 * the int8 C8 is requantised with the float fa/fb.  Both operands are packed
 * K-contiguous, then 64 x 64 blocks of C are computed from cache-resident
 * rows. */
static void gemm_i8(int transa, int transb, int m, int n, int k,
                    int32_t alpha, const int8_t *A, int lda,
                    const int8_t *B, int ldb, int32_t beta,
                    int32_t *C, int ldc, int8_t *C8, float fa, float fb) {
    int8_t *pa = pack_i8(transa, A, m, k, lda, 0);
    int8_t *pb = pack_i8(transb, B, n, k, ldb, 1);
    if (!pa || !pb) { free(pa); free(pb); return; }
    const int T = 64;
    const int bm = (m + T - 1) / T, bn = (n + T - 1) / T;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t blk = 0; blk < (int64_t)bm * bn; blk++) {
        const int i0 = (int)(blk % bm) * T, j0 = (int)(blk / bm) * T;
        const int i1 = i0 + T < m ? i0 + T : m, j1 = j0 + T < n ? j0 + T : n;
        for (int j = j0; j < j1; j++) {
            const int8_t *bj = pb + (size_t)j * k;
            for (int i = i0; i < i1; i++) {
                const uint32_t acc = dot_i8(pa + (size_t)i * k, bj, k);
                const int64_t at = i + (int64_t)j * ldc;
                if (C8) {
                    C8[at] = requant_s8((int32_t)acc, fa, fb, C8[at]);
                    continue;
                }
                uint32_t r = (uint32_t)alpha * acc;
                if (beta != 0)
                    r += (uint32_t)beta * (uint32_t)C[at];
                C[at] = (int32_t)r;
            }
        }
    }
    free(pa);
    free(pb);
}

/* fp64 dot product with four partial sums (fixed order: the result does
 * not depend on the host or the thread count). */
__attribute__((target_clones("arch=skylake-avx512", "avx2", "default")))
static double dot_f64(const double *a, const double *b, int k) {
    double s0 = 0.0, s1 = 0.0, s2 = 0.0, s3 = 0.0;
    int l = 0;
    for (; l + 4 <= k; l += 4) {
        s0 += a[l] * b[l];
        s1 += a[l + 1] * b[l + 1];
        s2 += a[l + 2] * b[l + 2];
        s3 += a[l + 3] * b[l + 3];
    }
    for (; l < k; l++) s0 += a[l] * b[l];
    return (s0 + s1) + (s2 + s3);
}

/* op(X) widened to a dense [rows][k] fp64 array (K contiguous), through
 * the reference converters. */
static double *pack_wide(int op, const void *X, int type, int rows, int k, int ld, int is_b) {
    double *p = malloc(sizeof(double) * (size_t)rows * (size_t)(k > 0 ? k : 1));
    if (!p) return NULL;
#pragma omp parallel for schedule(static)
    for (int r = 0; r < rows; r++)
        for (int l = 0; l < k; l++)
            p[(size_t)r * k + l] = is_b ? load_elem(X, type, opidx(op, l, r, ld))
                                        : load_elem(X, type, opidx(op, r, l, ld));
    return p;
}

/* 16-bit (or fp32) inputs, fp32 compute: restates gemm_ex_host
 * (zblas/zblas.c:318-356) -- widen, fp32 GEMM, narrow C.  The products are
 * summed in fp64 and rounded once to fp32 (at least as accurate as the
 * single-precision BLAS the reference calls), then narrowed with the
 * reference converter. */
static int gemm_wide(int transa, int transb, int m, int n, int k, float alpha,
                     const void *A, int Atype, int lda, const void *B, int Btype,
                     int ldb, float beta, void *C, int Ctype, int ldc) {
    double *pa = pack_wide(transa, A, Atype, m, k, lda, 0);
    double *pb = pack_wide(transb, B, Btype, n, k, ldb, 1);
    if (!pa || !pb) { free(pa); free(pb); return ZO_NOT_INITIALIZED; }
    const int T = 32;
    const int bm = (m + T - 1) / T, bn = (n + T - 1) / T;
#pragma omp parallel for schedule(dynamic, 1)
    for (int64_t blk = 0; blk < (int64_t)bm * bn; blk++) {
        const int i0 = (int)(blk % bm) * T, j0 = (int)(blk / bm) * T;
        const int i1 = i0 + T < m ? i0 + T : m, j1 = j0 + T < n ? j0 + T : n;
        for (int j = j0; j < j1; j++) {
            for (int i = i0; i < i1; i++) {
                double acc = dot_f64(pa + (size_t)i * k, pb + (size_t)j * k, k);
                int64_t at = i + (int64_t)j * ldc;
                double c = (double)alpha * acc;
                if (beta != 0.0f) c += (double)beta * load_elem(C, Ctype, at);
                float cf = (float)c;
                if (Ctype == ZO_R_16F) ((uint16_t *)C)[at] = zo_float_to_half(cf);
                else if (Ctype == ZO_R_16BF) ((uint16_t *)C)[at] = zo_float_to_bf16(cf);
                else ((float *)C)[at] = cf;
            }
        }
    }
    free(pa);
    free(pb);
    return ZO_OK;
}

/* The type/compute dispatch of cublasGemmEx (zblas/zblas.c:357-391), with
 * the int8 branch added.  alpha/beta are float* for 32F compute and
 * int32_t* for 32I compute. */
int zo_gemm_ex(int transa, int transb, int m, int n, int k, const void *alpha,
               const void *A, int Atype, int lda, const void *B, int Btype,
               int ldb, const void *beta, void *C, int Ctype, int ldc,
               int computeType) {
    if (Atype == ZO_R_8I && Btype == ZO_R_8I && Ctype == ZO_R_32I
        && (computeType == ZO_COMPUTE_32I || computeType == ZO_R_32I)) {
        gemm_i8(transa, transb, m, n, k, *(const int32_t *)alpha,
                (const int8_t *)A, lda, (const int8_t *)B, ldb,
                *(const int32_t *)beta, (int32_t *)C, ldc, NULL, 0.f, 0.f);
        return ZO_OK;
    }
    if (computeType != ZO_R_32F && computeType != ZO_COMPUTE_32F)
        return ZO_NOT_SUPPORTED;
    float al = *(const float *)alpha, be = *(const float *)beta;
    if (Atype == ZO_R_32F && Btype == ZO_R_32F && Ctype == ZO_R_32F) {
        zo_sgemm(transa, transb, m, n, k, al, (const float *)A, lda,
                 (const float *)B, ldb, be, (float *)C, ldc);
        return ZO_OK;
    }
    if (Atype == ZO_R_16BF && Btype == ZO_R_16BF) {
        /* gemm_ex_host(wide=1): C narrow iff Ctype is bf16, else fp32 */
        int ct = Ctype == ZO_R_16BF ? ZO_R_16BF : ZO_R_32F;
        return gemm_wide(transa, transb, m, n, k, al, A, Atype, lda, B, Btype,
                         ldb, be, C, ct, ldc);
    }
    if (Atype == ZO_R_16F && Btype == ZO_R_16F) {
        int ct = Ctype == ZO_R_16F ? ZO_R_16F : ZO_R_32F;
        return gemm_wide(transa, transb, m, n, k, al, A, Atype, lda, B, Btype,
                         ldb, be, C, ct, ldc);
    }
    return ZO_NOT_SUPPORTED;
}

/* cublasLtMatmul with int8 A/B/C/D, compute 32I and scale type 32F (no
 * counterpart in the reference): D = requant_s8(alpha * acc + beta * C),
 * float alpha/beta. */
int zo_gemm_i8_s8(int transa, int transb, int m, int n, int k, float alpha,
                  const int8_t *A, int lda, const int8_t *B, int ldb, float beta,
                  int8_t *C, int ldc) {
    gemm_i8(transa, transb, m, n, k, 0, A, lda, B, ldb, 0, NULL, ldc, C, alpha, beta);
    return ZO_OK;
}

static size_t zo_elem_size(int type) {
    switch (type) {
    case ZO_R_16F: case ZO_R_16BF: return 2;
    case ZO_R_8I: return 1;
    default: return 4;
    }
}

/* zblas/zblas.c:491-511.  The reference's elem_size (:488-490) returns 4
 * for every type that is not 16-bit; int8 is new here and uses 1. */
int zo_gemm_strided_batched_ex(int transa, int transb, int m, int n, int k,
                               const void *alpha, const void *A, int Atype,
                               int lda, long long sA, const void *B, int Btype,
                               int ldb, long long sB, const void *beta, void *C,
                               int Ctype, int ldc, long long sC, int batch,
                               int computeType) {
    for (int b = 0; b < batch; b++) {
        int rc = zo_gemm_ex(transa, transb, m, n, k, alpha,
                            (const char *)A + (size_t)b * sA * zo_elem_size(Atype),
                            Atype, lda,
                            (const char *)B + (size_t)b * sB * zo_elem_size(Btype),
                            Btype, ldb, beta,
                            (char *)C + (size_t)b * sC * zo_elem_size(Ctype),
                            Ctype, ldc, computeType);
        if (rc) return rc;
    }
    return ZO_OK;
}

/* Selected entries of C = alpha*op(A)op(B) + beta*C0 (no write to C):
 * out[t] for (rows[t], cols[t]), as fp64 before the final narrowing.  Used
 * to check full-size GEMMs by sampling. */
void zo_gemm_entries(int transa, int transb, int k, double alpha,
                     const void *A, int Atype, int lda,
                     const void *B, int Btype, int ldb, double beta,
                     const void *C0, int Ctype, int ldc,
                     const int64_t *rows, const int64_t *cols, int64_t count,
                     double *out) {
#pragma omp parallel for schedule(static)
    for (int64_t t = 0; t < count; t++) {
        int64_t i = rows[t], j = cols[t];
        double acc = 0.0;
        for (int l = 0; l < k; l++)
            acc += load_elem(A, Atype, opidx(transa, i, l, lda))
                 * load_elem(B, Btype, opidx(transb, l, j, ldb));
        double c = alpha * acc;
        if (beta != 0.0 && C0) c += beta * load_elem(C0, Ctype, i + j * (int64_t)ldc);
        out[t] = c;
    }
}

/* cublasLtMatmul's epilogue as the reference applies it after the GEMM
 * (zblas/zblas.c:692-710): D (already narrowed) is widened, bias[row] added
 * (bias in D's 16-bit type, fp32 otherwise), ReLU or tanh-form GELU applied
 * (zblas.c:638-642), and narrowed again.  flags: 1 bias, 2 relu, 4 gelu. */
static float zo_gelu_tanh(float x) {
    const float c = 0.7978845608028654f;
    float inner = c * (x + 0.044715f * x * x * x);
    return 0.5f * x * (1.0f + tanhf(inner));
}

void zo_lt_epilogue(void *D, int Dtype, int m, int n, int ldd, long long strideD, int batch,
                    const void *bias, int flags) {
    for (int b = 0; b < batch; b++) {
        for (int j = 0; j < n; j++) {
            for (int i = 0; i < m; i++) {
                int64_t at = (int64_t)b * strideD + i + (int64_t)j * ldd;
                float v = (float)load_elem(D, Dtype, at);
                if ((flags & 1) && bias) {
                    int bt = (Dtype == ZO_R_16F || Dtype == ZO_R_16BF) ? Dtype : ZO_R_32F;
                    v += (float)load_elem(bias, bt, i);
                }
                if ((flags & 2) && v < 0.0f) v = 0.0f;
                if (flags & 4) v = zo_gelu_tanh(v);
                if (Dtype == ZO_R_16F) ((uint16_t *)D)[at] = zo_float_to_half(v);
                else if (Dtype == ZO_R_16BF) ((uint16_t *)D)[at] = zo_float_to_bf16(v);
                else ((float *)D)[at] = v;
            }
        }
    }
}

/* ---- attention ------------------------------------------------------ */

typedef struct {
    const void *q, *k, *v;
    void *o;                       /* same element type as q/k/v */
    float *lse;                    /* [batch, heads, sq] fp32, may be NULL */
    int64_t qb, qh, qr, kb, kh, kr, vb, vh, vr, ob, oh, orr;  /* elements */
    int batch, heads, kv_ratio, sq, sk, d;
    float scale;
    int causal, diag;
    int elem;                      /* 0 = f16, 1 = bf16, 2 = f32 */
    const void *bias;              /* additive bias of the input type, may be NULL */
    int64_t bb, bh, br;            /* bias strides (elements) */
} zo_attn_desc;

static double ld_in(const void *p, int elem, int64_t at) {
    if (elem == 0) return zo_half_to_float(((const uint16_t *)p)[at]);
    if (elem == 1) return zo_bf16_to_float(((const uint16_t *)p)[at]);
    return ((const float *)p)[at];
}

static double round_in(double x, int elem) {
    if (elem == 0) return zo_half_to_float(zo_float_to_half((float)x));
    if (elem == 1) return zo_bf16_to_float(zo_float_to_bf16((float)x));
    return (float)x;
}

static void st_out(void *p, int elem, int64_t at, double x) {
    if (elem == 0) ((uint16_t *)p)[at] = zo_float_to_half((float)x);
    else if (elem == 1) ((uint16_t *)p)[at] = zo_float_to_bf16((float)x);
    else ((float *)p)[at] = (float)x;
}

/* One query row.  `work` holds sk doubles; `acc` holds d doubles.
 * Writes O (d elements) at the row's output address, and LSE if wanted.
 * If o_row is non-NULL it receives the fp64 O row before rounding. */
static void attn_row(const zo_attn_desc *p, int b, int h, int i,
                     double *work, double *acc, double *o_row, double *lse_row) {
    const int hk = h / p->kv_ratio;
    const int64_t qoff = b * p->qb + h * p->qh + (int64_t)i * p->qr;
    const int64_t koff = b * p->kb + hk * p->kh;
    const int64_t voff = b * p->vb + hk * p->vh;
    const int64_t ooff = b * p->ob + h * p->oh + (int64_t)i * p->orr;
    double mx = -INFINITY;
    for (int j = 0; j < p->sk; j++) {
        double s = 0.0;
        for (int t = 0; t < p->d; t++)
            s += ld_in(p->q, p->elem, qoff + t)
               * ld_in(p->k, p->elem, koff + (int64_t)j * p->kr + t);
        s *= (double)p->scale;
        /* bias added after scaling, before the mask (fmha_run :963-966,
         * fmha_f32 :822-823); read in its own type */
        if (p->bias)
            s += ld_in(p->bias, p->elem, b * p->bb + h * p->bh + (int64_t)i * p->br + j);
        if (p->causal && j > i + p->diag) s = -INFINITY;
        work[j] = s;
        if (s > mx) mx = s;
    }
    double sum = 0.0;
    for (int t = 0; t < p->d; t++) acc[t] = 0.0;
    for (int j = 0; j < p->sk; j++) {
        double e = mx == -INFINITY ? 0.0 : exp(work[j] - mx);
        sum += e;
        if (e == 0.0) continue;
        double pe = p->elem == 2 ? e : round_in(e, p->elem);
        for (int t = 0; t < p->d; t++)
            acc[t] += pe * ld_in(p->v, p->elem, voff + (int64_t)j * p->vr + t);
    }
    double inv = sum > 0.0 ? 1.0 / sum : 0.0;
    for (int t = 0; t < p->d; t++) {
        double o = acc[t] * inv;
        if (o_row) o_row[t] = o;
        if (p->o) st_out(p->o, p->elem, ooff + t, o);
    }
    double l = sum > 0.0 ? mx + log(sum) : -INFINITY;
    if (lse_row) *lse_row = l;
    if (p->lse)
        p->lse[((int64_t)b * p->heads + h) * p->sq + i] = (float)l;
}

/* Full attention forward over every (batch, head, query). */
int zo_attention(const zo_attn_desc *p) {
    if (!p || p->d <= 0 || p->sk <= 0 || p->kv_ratio <= 0) return ZO_INVALID_VALUE;
    const int64_t rows = (int64_t)p->batch * p->heads * p->sq;
#pragma omp parallel
    {
        double *work = malloc(sizeof(double) * (size_t)p->sk);
        double *acc = malloc(sizeof(double) * (size_t)p->d);
#pragma omp for schedule(dynamic, 16)
        for (int64_t r = 0; r < rows; r++) {
            int i = (int)(r % p->sq);
            int h = (int)((r / p->sq) % p->heads);
            int b = (int)(r / ((int64_t)p->sq * p->heads));
            attn_row(p, b, h, i, work, acc, NULL, NULL);
        }
        free(work);
        free(acc);
    }
    return ZO_OK;
}

/* Selected query rows only: for each t, (bs[t], hs[t], is[t]); writes the
 * fp64 O rows to o_rows[t*d ...] and the LSE to lse_rows[t].  Does not
 * touch p->o or p->lse. */
int zo_attention_rows(const zo_attn_desc *p, const int32_t *bs, const int32_t *hs,
                      const int32_t *is, int64_t count, double *o_rows,
                      double *lse_rows) {
    if (!p || p->d <= 0 || p->sk <= 0 || p->kv_ratio <= 0) return ZO_INVALID_VALUE;
    zo_attn_desc q = *p;
    q.o = NULL;
    q.lse = NULL;
#pragma omp parallel
    {
        double *work = malloc(sizeof(double) * (size_t)q.sk);
        double *acc = malloc(sizeof(double) * (size_t)q.d);
#pragma omp for schedule(dynamic, 1)
        for (int64_t t = 0; t < count; t++)
            attn_row(&q, bs[t], hs[t], is[t], work, acc, o_rows + t * q.d,
                     lse_rows + t);
        free(work);
        free(acc);
    }
    return ZO_OK;
}

int zo_attn_desc_size(void) { return (int)sizeof(zo_attn_desc); }
