// fmha.h -- internal description of one attention forward call, shared by
// the parameter-block decoders (attention_api.cu) and the kernel (fmha.cu).
// Mirrors the reference's AttnDesc (zblas/zblas_gpu.cpp:740-754).
#pragma once
#include <cuda_runtime.h>

namespace zl {

struct AttnDesc {
    const void *q, *k, *v;
    void* o;
    float* lse;                   // [batch][heads][sq] fp32, or null
    long long qb, qh, qr;         // batch / head / row strides, elements
    long long kb, kh, kr;
    long long vb, vh, vr;
    long long ob, oh, orr;
    int batches, heads, kv_ratio; // query head h reads K/V head h / kv_ratio
    int sq, sk, d;
    float scale;                  // applied to Q.K^T, natural-log units
    bool causal;
    int diag;                     // key j is masked for query i when j > i + diag
    int elem;                     // 0 fp16, 1 bf16, 2 fp32
    // Optional additive bias of the input type, added to the scaled scores
    // before the causal mask (zblas/zblas_gpu.cpp:963-966, :822-823):
    // bias[b*bb + h*bh + query*br + key], strides in elements.  Null: none.
    const void* bias;
    long long bb, bh, br;
    // Optional sub-range of (batch, head) pairs, for the partition layer:
    // the kernel covers pairs [pair_begin, pair_end) of batches*heads in
    // batch-major order.  pair_end == 0 means all.
    long long pair_begin, pair_end;
};

// 0 = enqueued, 1 = declined (shape/layout outside this kernel), > 1 = CUDA
// error code of the launch.
int fmha_fwd(const AttnDesc& d, cudaStream_t s);

// fp32 attention on the CUDA cores (elem == 2), same return convention.
int attn_f32_fwd(const AttnDesc& d, cudaStream_t s);

// Decodes a FlashAttention-2 parameter block and runs it (attention_api.cu);
// pair_end > 0 restricts it to (batch, head) pairs [pair_begin, pair_end).
int flash_entry(const void* params, unsigned bytes, int elem, cudaStream_t s,
                long long pair_begin, long long pair_end);

}  // namespace zl
