// gemm.h -- internal interface between the cuBLAS-style C ABI
// (cublas_api.cpp) and the GEMM kernels (gemm_tc.cu, gemm_simt.cu).
#pragma once
#include <cmath>
#include <cstdint>
#include <cuda_runtime.h>

namespace zl {

// cudaDataType_t values used at the boundary (same numbers as CUDA's).
enum DType : int {
    kR32F = 0,
    kR16F = 2,
    kR8I = 3,
    kR32I = 10,
    kR16BF = 14,
};

// How the tensor cores consume the inputs.
enum class Kind : int {
    F16 = 0,      // kind::f16, fp16 inputs
    BF16 = 1,     // kind::f16, bf16 inputs
    TF32X3 = 2,   // fp32 inputs as hi+lo tf32 planes, 3 products
    TF32 = 3,     // fp32 inputs, one tf32 product (CUBLAS_TF32_TENSOR_OP_MATH)
    I8 = 4,       // kind::i8, int32 accumulate
};

// One (possibly batched) column-major GEMM:
//   C[b] = alpha * op(A[b]) * op(B[b]) + beta * C[b],  b < batch.
// Strides and leading dimensions are in elements.  alpha/beta are read
// from the host values unless the *_dev pointers are set (device pointer
// mode), in which case the kernel dereferences them.
struct GemmDesc {
    int transa, transb;          // 0 = N, 1 = T (2 = C is treated as T)
    int m, n, k, batch;
    const void* A; long long lda, strideA; int Atype;
    const void* B; long long ldb, strideB; int Btype;
    void* C; long long ldc, strideC; int Ctype;
    Kind kind;
    float alpha, beta;           // 32F compute
    int32_t ialpha, ibeta;       // 32I compute
    const void* alpha_dev;       // device pointer mode (float* or int32_t*)
    const void* beta_dev;
    // fp32 split planes for Kind::TF32X3: hi and lo copies of A and B with
    // the same layout as A and B.  Filled by the caller through split_tf32.
    const float* A_lo; const float* B_lo;
    const float* A_hi; const float* B_hi;
    // Fused epilogue after alpha*acc + beta*C (floating-point outputs only):
    // kEpiBias adds bias[row] (a length-m vector of bias_type), then kEpiRelu
    // or kEpiGelu (tanh form) is applied.
    int epi;
    const void* bias;
    int bias_type;
    // Workspace for splitting the last wave of tiles along K (null: never
    // split): split_work_bytes of device memory for partial sums and one
    // counter per split tile and CTA (at most 2 * number of SMs), zero on
    // first use.  split_epoch tags the launch (a different value per launch
    // that shares the workspace, nonzero, < 2^48).
    uint32_t* split_work = nullptr;
    size_t split_work_bytes = 0;
    unsigned long long* split_counters = nullptr;
    unsigned long long split_epoch = 0;
    // Most SMs the persistent kernel may occupy (0 = all; cublasSetSmCountTarget),
    // e.g. to leave SMs to a collective that runs at the same time.
    int sm_limit = 0;
};

enum EpiFlags : int { kEpiBias = 1, kEpiRelu = 2, kEpiGelu = 4 };

// int8 output of an int32 accumulator with float scaling (cuBLASLt's int8 D
// with a 32F scale type): x = alpha * float(acc) (+ beta * float(C)), then
// rounded to nearest with ties to even and saturated to [-128, 127]; NaN
// gives 0.  The float steps are explicit (one rounded multiply, one fused
// multiply-add) so that a CPU restatement reproduces every bit.
__device__ __forceinline__ int8_t requant_s8(int32_t acc, float alpha, bool use_beta, float beta,
                                             int8_t old) {
    float x = __fmul_rn(alpha, __int2float_rn(acc));
    if (use_beta) x = __fmaf_rn(beta, __int2float_rn((int)old), x);
    if (x != x) return 0;
    const int r = __float2int_rn(x);
    return (int8_t)(r < -128 ? -128 : (r > 127 ? 127 : r));
}

// x after the fused epilogue (bias already added by the caller if requested)
__host__ __device__ inline float apply_act(float x, int epi) {
    if (epi & kEpiRelu) x = x > 0.f ? x : 0.f;
    if (epi & kEpiGelu) {
        const float u = 0.7978845608028654f * (x + 0.044715f * x * x * x);
        x = 0.5f * x * (1.f + tanhf(u));
    }
    return x;
}

// Tensor-core path.  Returns 0 when launched, 1 when this shape/layout is
// not eligible (the caller then uses the general kernel), or a CUDA error
// code (> 1) on a launch failure.
int gemm_tc(const GemmDesc& d, cudaStream_t s);

// General CUDA-core kernel: any shape, any leading dimension, any alignment.
int gemm_simt(const GemmDesc& d, cudaStream_t s);

// Split an fp32 operand into K-major tf32 planes hi = rn(x), lo = rn(x - hi)
// (round to nearest, ties away, to tf32's 10 mantissa bits).  Element
// (mn, l), mn < MN, l < K, is read from X[b*stride + (k_contig ? mn*ld + l :
// l*ld + mn)] and written to plane[b*MN*kp + mn*kp + l]; columns K..kp-1
// are zero.  lo may be null (one-product tf32 mode).
int split_tf32(const float* X, bool k_contig, long long MN, long long K, long long ld,
               long long stride, int batch, long long kp, float* hi, float* lo,
               cudaStream_t s);

// fp64 GEMM on the CUDA cores (column-major, op 0 = N, 1 = T/C); alpha and
// beta from the host values unless the *_dev pointers are set.
int dgemm_simt(int transa, int transb, int m, int n, int k, double alpha, double beta,
               const double* alpha_dev, const double* beta_dev, const double* A, long long lda,
               const double* B, long long ldb, double* C, long long ldc, cudaStream_t s);

int num_sms();

// Count of kernels this library has launched (all devices, all streams).
void note_launch(unsigned n = 1);
unsigned long long launch_count();

// Device error words of the kernel translation units (read, optionally clear).
int gemm_tc_error(bool clear);
int gemm_tc_set_wait_limit(unsigned long long ns);
int gemm_simt_set_wait_limit(unsigned long long ns);
int fmha_set_wait_limit(unsigned long long ns);
int part_error(bool clear);
int part_set_wait_limit(unsigned long long ns);
unsigned long long wait_limit_ns();
// Launches a one-thread kernel whose mbarrier wait nobody completes: it
// gives up after limit_ns, records kErrWaitTimeout and returns.
int wait_probe(unsigned long long limit_ns, cudaStream_t s);
int gemm_simt_error(bool clear);
int fmha_error(bool clear);

// Trace switch (ZBLAS_TRACE set in the environment).
bool tracing();

}  // namespace zl
