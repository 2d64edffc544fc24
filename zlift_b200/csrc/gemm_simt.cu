// gemm_simt.cu -- the general CUDA-core GEMM and the fp32 -> tf32 split.
//
// gemm_simt answers every GEMM the tensor-core path declines: leading
// dimensions or base addresses that TMA cannot describe (not 16-byte
// aligned), k == 0, and very small shapes.  It plays the part the
// reference gives its CPU fallback (zblas/zblas.c:127, :344), on the GPU.
// Accumulation: fp32 FMA for floating types, exact int32 for int8.
//
// split_tf32 writes hi = rn_tf32(x) and lo = rn_tf32(x - hi) planes for the
// 3-product fp32 path; it replaces the reference's split_to_bf16
// (zblas/zblas_gpu.cpp:219-265), which splits into bf16 planes instead.
#include "gemm.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace zl {

namespace {

constexpr int TS = 32;        // output tile edge
constexpr int KS = 16;        // K slice held in shared memory

struct SimtParams {
    int transa, transb, m, n, k;
    const void* A; long long lda, sA; int At;
    const void* B; long long ldb, sB; int Bt;
    void* C; long long ldc, sC; int Ct;
    float alpha, beta;
    int32_t ia, ib;
    const void* alpha_dev;
    const void* beta_dev;
    int epi;
    const void* bias;
    int bias_type;
};

__device__ __forceinline__ float ldf(const void* p, int t, long long at) {
    switch (t) {
    case kR16F: return __half2float(static_cast<const __half*>(p)[at]);
    case kR16BF: return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[at]);
    case kR8I: return (float)static_cast<const int8_t*>(p)[at];
    default: return static_cast<const float*>(p)[at];
    }
}

// element (i, l) of op(X)
__device__ __forceinline__ long long opidx(int op, long long i, long long l, long long ld) {
    return op == 0 ? i + l * ld : l + i * ld;
}

// 32x32 output tile per 256 threads (each thread 4 outputs in a column).
template <bool INT>
__global__ void __launch_bounds__(256) gemm_simt_kernel(const SimtParams p) {
    __shared__ float sa[KS][TS + 1];
    __shared__ float sb[KS][TS + 1];
    __shared__ int sai[INT ? KS : 1][TS + 1];
    __shared__ int sbi[INT ? KS : 1][TS + 1];
    const int bz = blockIdx.z;
    const char* A = static_cast<const char*>(p.A);
    const char* B = static_cast<const char*>(p.B);
    const int ea = p.At == kR8I ? 1 : (p.At == kR16F || p.At == kR16BF) ? 2 : 4;
    const int eb = p.Bt == kR8I ? 1 : (p.Bt == kR16F || p.Bt == kR16BF) ? 2 : 4;
    A += (long long)bz * p.sA * ea;
    B += (long long)bz * p.sB * eb;
    const int i0 = blockIdx.x * TS, j0 = blockIdx.y * TS;
    const int tx = threadIdx.x & 31;       // row within tile
    const int ty = threadIdx.x >> 5;       // 0..7 -> columns ty, ty+8, ty+16, ty+24
    float acc[4] = {0.f, 0.f, 0.f, 0.f};
    int iacc[4] = {0, 0, 0, 0};
    for (int l0 = 0; l0 < p.k; l0 += KS) {
        for (int e = threadIdx.x; e < KS * TS; e += 256) {
            const int r = e % TS, l = e / TS;
            const long long gi = i0 + r, gl = l0 + l, gj = j0 + r;
            if constexpr (INT) {
                sai[l][r] = (gi < p.m && gl < p.k)
                    ? (int)static_cast<const int8_t*>((const void*)A)[opidx(p.transa, gi, gl, p.lda)] : 0;
                sbi[l][r] = (gj < p.n && gl < p.k)
                    ? (int)static_cast<const int8_t*>((const void*)B)[opidx(p.transb, gl, gj, p.ldb)] : 0;
            } else {
                sa[l][r] = (gi < p.m && gl < p.k) ? ldf(A, p.At, opidx(p.transa, gi, gl, p.lda)) : 0.f;
                sb[l][r] = (gj < p.n && gl < p.k) ? ldf(B, p.Bt, opidx(p.transb, gl, gj, p.ldb)) : 0.f;
            }
        }
        __syncthreads();
#pragma unroll
        for (int l = 0; l < KS; l++) {
#pragma unroll
            for (int c = 0; c < 4; c++) {
                if constexpr (INT) iacc[c] += sai[l][tx] * sbi[l][ty + 8 * c];
                else acc[c] = fmaf(sa[l][tx], sb[l][ty + 8 * c], acc[c]);
            }
        }
        __syncthreads();
    }
    float alpha = p.alpha, beta = p.beta;
    int32_t ia = p.ia, ib = p.ib;
    // int32 scalars for int32 C; float for every other output (int8 C is
    // requantised with float scaling)
    const bool iscale = INT && p.Ct == kR32I;
    if (p.alpha_dev) {
        if (iscale) ia = *static_cast<const int32_t*>(p.alpha_dev);
        else alpha = *static_cast<const float*>(p.alpha_dev);
    }
    if (p.beta_dev) {
        if (iscale) ib = *static_cast<const int32_t*>(p.beta_dev);
        else beta = *static_cast<const float*>(p.beta_dev);
    }
    const long long gi = i0 + tx;
    if (gi >= p.m) return;
    const float bias_row = (p.epi & kEpiBias) && p.bias ? ldf(p.bias, p.bias_type, gi) : 0.f;
#pragma unroll
    for (int c = 0; c < 4; c++) {
        const long long gj = j0 + ty + 8 * c;
        if (gj >= p.n) continue;
        const long long at = (long long)bz * p.sC + gi + gj * p.ldc;
        if constexpr (INT) {
            if (p.Ct == kR8I) {
                int8_t* cp = static_cast<int8_t*>(p.C) + at;
                *cp = requant_s8(iacc[c], alpha, beta != 0.f, beta, beta != 0.f ? *cp : 0);
            } else {
                int32_t* cp = static_cast<int32_t*>(p.C) + at;
                uint32_t v = (uint32_t)ia * (uint32_t)iacc[c];
                if (ib != 0) v += (uint32_t)ib * (uint32_t)(*cp);
                *cp = (int32_t)v;
            }
        } else {
            float v = alpha * acc[c];
            if (p.Ct == kR16F) {
                __half* cp = static_cast<__half*>(p.C) + at;
                if (beta != 0.f) v = fmaf(beta, __half2float(*cp), v);
                if (p.epi) v = apply_act(v + bias_row, p.epi);
                *cp = __float2half_rn(v);
            } else if (p.Ct == kR16BF) {
                __nv_bfloat16* cp = static_cast<__nv_bfloat16*>(p.C) + at;
                if (beta != 0.f) v = fmaf(beta, __bfloat162float(*cp), v);
                if (p.epi) v = apply_act(v + bias_row, p.epi);
                *cp = __float2bfloat16_rn(v);
            } else {
                float* cp = static_cast<float*>(p.C) + at;
                if (beta != 0.f) v = fmaf(beta, *cp, v);
                if (p.epi) v = apply_act(v + bias_row, p.epi);
                *cp = v;
            }
        }
    }
}

__device__ __forceinline__ float tf32_rn(float x) {
    uint32_t r;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
    return __uint_as_float(r);
}

// Element (mn, l) of the operand (mn < MN, l < K) is read from
// X[b*stride + (k_contig ? mn*ld + l : l*ld + mn)] and written K-major to
// hi/lo[b*MN*kp + mn*kp + l].  32x32 tiles go through shared memory so both
// the read (along the source's contiguous dimension) and the write (along
// K) are coalesced.  lo may be null (one tf32 product).
__global__ void __launch_bounds__(256)
split_tf32_kernel(const float* __restrict__ X, int k_contig, long long MN, long long K,
                  long long ld, long long stride, long long kp,
                  float* __restrict__ hi, float* __restrict__ lo) {
    __shared__ float tile[32][33];
    const long long b = blockIdx.z;
    const long long mn0 = (long long)blockIdx.y * 32, l0 = (long long)blockIdx.x * 32;
    const float* src = X + b * stride;
    const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;   // 32 x 8
    for (int r = ty; r < 32; r += 8) {
        // k_contig: tile[mn][l] read along l; else tile[mn][l] read along mn
        long long mn, l;
        if (k_contig) { mn = mn0 + r; l = l0 + tx; }
        else { mn = mn0 + tx; l = l0 + r; }
        float v = 0.f;
        if (mn < MN && l < K) v = src[k_contig ? mn * ld + l : l * ld + mn];
        if (k_contig) tile[r][tx] = v;
        else tile[tx][r] = v;
    }
    __syncthreads();
    float* dh = hi + b * MN * kp;
    float* dl = lo ? lo + b * MN * kp : nullptr;
    for (int r = ty; r < 32; r += 8) {
        const long long mn = mn0 + r, l = l0 + tx;
        if (mn < MN && l < kp) {
            const float x = l < K ? tile[r][tx] : 0.f;
            const float h = tf32_rn(x);
            dh[mn * kp + l] = h;
            if (dl) dl[mn * kp + l] = tf32_rn(x - h);
        }
    }
}

}  // namespace

int gemm_simt(const GemmDesc& d, cudaStream_t s) {
    if (d.m <= 0 || d.n <= 0 || d.batch <= 0) return 0;
    SimtParams p;
    p.transa = d.transa; p.transb = d.transb;
    p.m = d.m; p.n = d.n; p.k = d.k;
    p.A = d.A; p.lda = d.lda; p.sA = d.strideA; p.At = d.Atype;
    p.B = d.B; p.ldb = d.ldb; p.sB = d.strideB; p.Bt = d.Btype;
    p.C = d.C; p.ldc = d.ldc; p.sC = d.strideC; p.Ct = d.Ctype;
    p.alpha = d.alpha; p.beta = d.beta;
    p.ia = d.ialpha; p.ib = d.ibeta;
    p.alpha_dev = d.alpha_dev; p.beta_dev = d.beta_dev;
    p.epi = d.kind == Kind::I8 ? 0 : d.epi;
    p.bias = d.bias;
    p.bias_type = d.bias_type;
    dim3 grid((d.m + TS - 1) / TS, (d.n + TS - 1) / TS, d.batch);
    if (grid.y > 65535u || grid.z > 65535u) return 1;
    if (d.kind == Kind::I8) gemm_simt_kernel<true><<<grid, 256, 0, s>>>(p);
    else gemm_simt_kernel<false><<<grid, 256, 0, s>>>(p);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

int split_tf32(const float* X, bool k_contig, long long MN, long long K, long long ld,
               long long stride, int batch, long long kp, float* hi, float* lo,
               cudaStream_t s) {
    if (MN <= 0 || K <= 0 || batch <= 0) return 0;
    const long long gx = (kp + 31) / 32, gy = (MN + 31) / 32;
    if (gx > 0x7fffffffLL || gy > 65535 || batch > 65535) return 1;
    dim3 grid((unsigned)gx, (unsigned)gy, (unsigned)batch);
    split_tf32_kernel<<<grid, 256, 0, s>>>(X, k_contig ? 1 : 0, MN, K, ld, stride, kp, hi, lo);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

namespace {

// fp64 GEMM (cublasDgemm_v2; the reference hands it to oneMKL on the GPU,
// zblas/zblas_gpu.cpp:1548-1559, or cblas_dgemm on the host,
// zblas/zblas.c:131-144).  64 x 64 output tile per 256 threads, each thread
// a 4 x 4 block (rows ty*4.., columns tx + 16c), K in slices of 16 through
// shared memory; fp64 FMA in K order.
constexpr int DT = 64, DK = 16;

__global__ void __launch_bounds__(256) dgemm_kernel(int transa, int transb, int m, int n, int k,
                                                    double alpha, double beta,
                                                    const double* alpha_dev,
                                                    const double* beta_dev,
                                                    const double* __restrict__ A, long long lda,
                                                    const double* __restrict__ B, long long ldb,
                                                    double* __restrict__ C, long long ldc) {
    __shared__ double sa[DK][DT + 1];
    __shared__ double sb[DK][DT + 1];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int i0 = blockIdx.x * DT, j0 = blockIdx.y * DT;
    double acc[4][4] = {};
    for (int l0 = 0; l0 < k; l0 += DK) {
        for (int e = threadIdx.x; e < DK * DT; e += 256) {
            // transa == N reads down a column (i fastest): coalesced for N,
            // strided for T
            const int r = transa == 0 ? e % DT : e / DK, l = transa == 0 ? e / DT : e % DK;
            const long long gi = i0 + r, gl = l0 + l;
            sa[l][r] = (gi < m && gl < k) ? A[opidx(transa, gi, gl, lda)] : 0.0;
        }
        for (int e = threadIdx.x; e < DK * DT; e += 256) {
            const int c = transb == 0 ? e / DK : e % DT, l = transb == 0 ? e % DK : e / DT;
            const long long gj = j0 + c, gl = l0 + l;
            sb[l][c] = (gj < n && gl < k) ? B[opidx(transb, gl, gj, ldb)] : 0.0;
        }
        __syncthreads();
#pragma unroll
        for (int l = 0; l < DK; l++) {
            double a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; i++) a[i] = sa[l][ty * 4 + i];
#pragma unroll
            for (int c = 0; c < 4; c++) b[c] = sb[l][tx + 16 * c];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int c = 0; c < 4; c++) acc[i][c] = fma(a[i], b[c], acc[i][c]);
        }
        __syncthreads();
    }
    if (alpha_dev) alpha = *alpha_dev;
    if (beta_dev) beta = *beta_dev;
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const long long gi = i0 + ty * 4 + i;
        if (gi >= m) continue;
#pragma unroll
        for (int c = 0; c < 4; c++) {
            const long long gj = j0 + tx + 16 * c;
            if (gj >= n) continue;
            double* cp = C + gi + gj * ldc;
            // beta == 0 does not read C (BLAS convention)
            *cp = beta != 0.0 ? fma(beta, *cp, alpha * acc[i][c]) : alpha * acc[i][c];
        }
    }
}

}  // namespace

int dgemm_simt(int transa, int transb, int m, int n, int k, double alpha, double beta,
               const double* alpha_dev, const double* beta_dev, const double* A, long long lda,
               const double* B, long long ldb, double* C, long long ldc, cudaStream_t s) {
    if (m <= 0 || n <= 0) return 0;
    const long long gx = (m + DT - 1) / DT, gy = (n + DT - 1) / DT;
    if (gx > 0x7fffffffLL || gy > 65535) return 1;
    dgemm_kernel<<<dim3((unsigned)gx, (unsigned)gy), 256, 0, s>>>(
        transa, transb, m, n, k, alpha, beta, alpha_dev, beta_dev, A, lda, B, ldb, C, ldc);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

// A wait that nothing completes: one thread initialises an mbarrier that
// expects one arrival and waits on its first phase with `limit_ns`.  No
// copy or MMA is in flight, so the kernel simply returns after the limit,
// with kErrWaitTimeout in this unit's error word.
__global__ void wait_probe_kernel(unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_mbar_init();
        mbar_wait_for(&bar, 0, &abort_flag, limit_ns);
    }
}

int wait_probe(unsigned long long limit_ns, cudaStream_t s) {
    wait_probe_kernel<<<1, 32, 0, s>>>(limit_ns);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

unsigned long long wait_limit_ns() { return get_unit_wait_limit(); }

int gemm_simt_set_wait_limit(unsigned long long ns) { return set_unit_wait_limit(ns); }

int gemm_simt_error(bool clear) {
    int v = 0;
    cudaMemcpyFromSymbol(&v, g_dev_error, sizeof(int));
    if (clear && v) {
        int z = 0;
        cudaMemcpyToSymbol(g_dev_error, &z, sizeof(int));
    }
    return v;
}

}  // namespace zl
