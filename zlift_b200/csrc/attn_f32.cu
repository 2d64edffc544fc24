// attn_f32.cu -- fp32 attention forward on the CUDA cores.
//
// Serves the reference's fp32 attention (elem == 2, attn_dispatch
// zblas/zblas_gpu.cpp:1367-1372), whose math is fmha_f32 (:793-844):
// s = (q . k) * scale (+ bias), causal mask `key > query + diag`, softmax
// with exp in fp32, O = sum_j softmax_j * v_j; a fully masked row gives
// O = 0.  The reference materialises the whole score matrix in a scratch
// buffer (and declines calls above 16M scores, :1399-1406); this kernel is
// a flash-style online softmax over key tiles instead, so it needs no
// scratch and has no size limit, and it also writes the log-sum-exp when
// asked (natural log, m + ln l).
//
// One CTA = 64 queries of one (batch, head), 256 threads as 16 x 16: thread
// (ty, tx) owns query rows 4ty..4ty+3 and, per 64-key tile, keys tx + 16c
// (c < 4) of S and output columns tx + 16c (c < ceil(D/16)) of O.  Q, K, V
// and P tiles live in shared memory with odd row strides (no bank
// conflicts).  head_dim 1..256.
#include "fmha.h"
#include "gemm.h"

#include <cmath>

namespace zl {

namespace {

constexpr int TQ = 64;       // queries per CTA
constexpr int TK = 64;       // keys per tile
constexpr int kMaxD = 256;

template <int DC>            // DC = ceil(D / 16) output columns per thread
__global__ void __launch_bounds__(256)
attn_f32_kernel(const float* __restrict__ q, const float* __restrict__ k,
                const float* __restrict__ v, float* __restrict__ o, float* __restrict__ lse,
                const float* __restrict__ bias, AttnDesc d, long long bh0) {
    extern __shared__ float sm[];
    const int D = d.d, ld = D + 1;             // odd row stride
    float* sq = sm;                            // [TQ][ld]
    float* sk = sq + TQ * ld;                  // [TK][ld]
    float* sv = sk + TK * ld;                  // [TK][ld]
    float* sp = sv + TK * ld;                  // [TQ][TK + 1]
    const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
    const int q0 = blockIdx.x * TQ;
    const long long bh = bh0 + blockIdx.y;
    const int b = (int)(bh / d.heads), h = (int)(bh % d.heads), hk = h / d.kv_ratio;
    const float* qb = q + b * d.qb + h * d.qh;
    const float* kb = k + b * d.kb + hk * d.kh;
    const float* vb = v + b * d.vb + hk * d.vh;
    const float* biasb = bias ? bias + b * d.bb + h * d.bh : nullptr;

    for (int i = tid; i < TQ * D; i += 256) {
        const int r = i / D, c = i - r * D;
        sq[r * ld + c] = q0 + r < d.sq ? qb[(long long)(q0 + r) * d.qr + c] : 0.f;
    }
    float m[4], l[4], acc[4][DC];
#pragma unroll
    for (int i = 0; i < 4; i++) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int c = 0; c < DC; c++) acc[i][c] = 0.f;
    }
    // key tiles this query tile needs (causal: up to its last query's diagonal)
    int kend = d.sk;
    if (d.causal) {
        const long long last = (long long)min(q0 + TQ - 1, d.sq - 1) + d.diag;
        kend = last < 0 ? 0 : (int)min((long long)d.sk, last + 1);
    }
    for (int k0 = 0; k0 < kend; k0 += TK) {
        __syncthreads();       // previous tile's K, V and P are no longer read
        for (int i = tid; i < TK * D; i += 256) {
            const int r = i / D, c = i - r * D;
            const bool in = k0 + r < d.sk;
            sk[r * ld + c] = in ? kb[(long long)(k0 + r) * d.kr + c] : 0.f;
            sv[r * ld + c] = in ? vb[(long long)(k0 + r) * d.vr + c] : 0.f;
        }
        __syncthreads();
        float s[4][4];
#pragma unroll
        for (int i = 0; i < 4; i++)
#pragma unroll
            for (int c = 0; c < 4; c++) s[i][c] = 0.f;
        for (int e = 0; e < D; e++) {
            float qa[4], ka[4];
#pragma unroll
            for (int i = 0; i < 4; i++) qa[i] = sq[(4 * ty + i) * ld + e];
#pragma unroll
            for (int c = 0; c < 4; c++) ka[c] = sk[(tx + 16 * c) * ld + e];
#pragma unroll
            for (int i = 0; i < 4; i++)
#pragma unroll
                for (int c = 0; c < 4; c++) s[i][c] = fmaf(qa[i], ka[c], s[i][c]);
        }
        // scale, bias, mask; online softmax per row (rows are shared by the
        // 16 lanes tx of a half-warp)
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int qi = q0 + 4 * ty + i;
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const int key = k0 + tx + 16 * c;
                float x = s[i][c] * d.scale;
                if (biasb && key < d.sk && qi < d.sq) x += biasb[(long long)qi * d.br + key];
                if (key >= d.sk || (d.causal && key > qi + d.diag)) x = -INFINITY;
                s[i][c] = x;
                mx = fmaxf(mx, x);
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            float sum = 0.f;
#pragma unroll
            for (int c = 0; c < 4; c++) {
                const float pe = mn == -INFINITY ? 0.f : expf(s[i][c] - mn);
                sum += pe;
                sp[(4 * ty + i) * (TK + 1) + tx + 16 * c] = pe;
            }
#pragma unroll
            for (int off = 8; off > 0; off >>= 1)
                sum += __shfl_xor_sync(0xffffffffu, sum, off);
            const float corr = mn == -INFINITY ? 0.f : expf(m[i] - mn);
            l[i] = l[i] * corr + sum;
            m[i] = mn;
#pragma unroll
            for (int c = 0; c < DC; c++) acc[i][c] *= corr;
        }
        __syncthreads();
        const int kn = min(TK, d.sk - k0);
        for (int j = 0; j < kn; j++) {
            float pv[4];
#pragma unroll
            for (int i = 0; i < 4; i++) pv[i] = sp[(4 * ty + i) * (TK + 1) + j];
#pragma unroll
            for (int c = 0; c < DC; c++) {
                const int col = tx + 16 * c;
                const float vv = col < D ? sv[j * ld + col] : 0.f;
#pragma unroll
                for (int i = 0; i < 4; i++) acc[i][c] = fmaf(pv[i], vv, acc[i][c]);
            }
        }
    }
#pragma unroll
    for (int i = 0; i < 4; i++) {
        const int qi = q0 + 4 * ty + i;
        if (qi >= d.sq) continue;
        const float inv = l[i] > 0.f ? 1.f / l[i] : 0.f;
        float* orow = o + b * d.ob + h * d.oh + (long long)qi * d.orr;
#pragma unroll
        for (int c = 0; c < DC; c++) {
            const int col = tx + 16 * c;
            if (col < D) orow[col] = acc[i][c] * inv;
        }
        if (lse && tx == 0)
            lse[bh * (long long)d.sq + qi] = l[i] > 0.f ? m[i] + logf(l[i]) : -INFINITY;
    }
}

template <int DC>
int launch_f32(const AttnDesc& d, long long bh0, long long nbh, cudaStream_t s) {
    const size_t smem = sizeof(float) * ((size_t)(TQ + 2 * TK) * (d.d + 1) + TQ * (TK + 1));
    auto kern = attn_f32_kernel<DC>;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             (int)smem);
        if (e != cudaSuccess) return (int)e;
    }
    dim3 grid((unsigned)((d.sq + TQ - 1) / TQ), (unsigned)nbh);
    kern<<<grid, 256, smem, s>>>(static_cast<const float*>(d.q), static_cast<const float*>(d.k),
                                 static_cast<const float*>(d.v), static_cast<float*>(d.o), d.lse,
                                 static_cast<const float*>(d.bias), d, bh0);
    cudaError_t e = cudaGetLastError();
    if (e == cudaSuccess) note_launch();
    return e == cudaSuccess ? 0 : (int)e;
}

}  // namespace

int attn_f32_fwd(const AttnDesc& d, cudaStream_t s) {
    if (d.elem != 2) return 1;
    if (d.d <= 0 || d.d > kMaxD) return 1;
    if (d.batches <= 0 || d.heads <= 0 || d.sq <= 0 || d.sk <= 0 || d.kv_ratio <= 0) return 1;
    if (d.heads % d.kv_ratio) return 1;
    const long long total = (long long)d.batches * d.heads;
    const long long bh0 = d.pair_end > 0 ? d.pair_begin : 0;
    const long long nbh = d.pair_end > 0 ? d.pair_end - d.pair_begin : total;
    if (nbh <= 0) return 0;
    if (nbh > 65535) return 1;
    const int dc = (d.d + 15) / 16;
    if (dc <= 2) return launch_f32<2>(d, bh0, nbh, s);
    if (dc <= 4) return launch_f32<4>(d, bh0, nbh, s);
    if (dc <= 8) return launch_f32<8>(d, bh0, nbh, s);
    return launch_f32<16>(d, bh0, nbh, s);
}

}  // namespace zl
