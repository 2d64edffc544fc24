// attention_api.cu -- decoders for the two attention parameter blocks the
// reference accepts (zblas/zblas_gpu.cpp:1424-1535), mapped onto one
// internal AttnDesc and the fused forward kernel in fmha.cu.
//
// The validation follows the reference's checks line by line (same
// declines, same meaning of every field), with these differences:
//   - an LSE pointer is honoured instead of ignored (flash) or declined
//     (xformers);
//   - fp32 inputs (elem 2) run on attn_f32.cu's flash-style CUDA-core kernel,
//     which needs no score scratch, so the reference's 16M-score limit
//     (attn_tiles, zblas_gpu.cpp:1399-1406) does not apply;
//   - the kernels' own layout limits (tensor cores: head_dim 64 or 128,
//     16-byte aligned rows; fp32: head_dim up to 256) replace the reference's
//     tile limits (attn_tiles :1398-1423).
#include "fmha.h"
#include "gemm.h"

#include "../../include/zlift_attention.h"

#include <cstddef>
#include <cstdio>
#include <cstring>

static_assert(offsetof(zlift_flash_params, h) == 96, "flash params layout");
static_assert(offsetof(zlift_flash_params, o_ptr) == 112, "flash params layout");
static_assert(offsetof(zlift_flash_params, p_ptr) == 152, "flash params layout");
static_assert(offsetof(zlift_flash_params, softmax_lse_ptr) == 160, "flash params layout");
static_assert(offsetof(zlift_flash_params, b) == 176, "flash params layout");
static_assert(offsetof(zlift_flash_params, scale_softmax) == 216, "flash params layout");
static_assert(offsetof(zlift_flash_params, opaque) == 224, "flash params layout");
static_assert(offsetof(zlift_flash_params, p_dropout) == 372, "flash params layout");
static_assert(offsetof(zlift_flash_params, rp_dropout) == 380, "flash params layout");
static_assert(offsetof(zlift_flash_params, window_size_left) == 388, "flash params layout");
static_assert(offsetof(zlift_fmha_params, output_ptr) == 64, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, scale) == 92, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, num_queries) == 104, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, custom_mask_type) == 116, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, q_strideM) == 120, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, bias_strideH) == 152, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, num_batches) == 192, "fmha params layout");
static_assert(offsetof(zlift_fmha_params, use_dropout) == 200, "fmha params layout");

namespace {

cudaStream_t g_attn_stream = nullptr;

int declined(const char* who, const char* why) {
    if (zl::tracing()) fprintf(stderr, "[zblas] %s declined: %s\n", who, why);
    return 1;
}

int run(const char* who, const zl::AttnDesc& d, cudaStream_t s) {
    int rc = zl::fmha_fwd(d, s);
    if (rc == 1) return declined(who, "shape or layout outside the fused kernel");
    if (rc != 0) {
        if (zl::tracing()) fprintf(stderr, "[zblas] %s launch failed: %d\n", who, rc);
        cudaGetLastError();
        return 2;
    }
    if (zl::tracing())
        fprintf(stderr, "[zblas] %s %s %dx%d heads %d keys %d dim %d%s\n", who,
                d.elem == 2 ? "f32" : d.elem == 1 ? "bf16" : "f16", d.batches, d.sq, d.heads,
                d.sk, d.d, d.bias ? " bias" : "");
    return 0;
}

}  // namespace

namespace zl {

// zblas/zblas_gpu.cpp:1477-1535.  pair_end > 0 restricts the call to
// (batch, head) pairs [pair_begin, pair_end) (partition layer).
int flash_entry(const void* params, unsigned bytes, int elem, cudaStream_t s,
                long long pair_begin, long long pair_end) {
    const char* who = "flash";
    if (!params || bytes < ZLIFT_FLASH_PARAMS_BYTES) return 1;
    const unsigned char* raw = static_cast<const unsigned char*>(params);
    zlift_flash_params p;
    std::memcpy(&p, params, sizeof p);
    auto zeroes = [&](unsigned from, unsigned to) {
        for (unsigned i = from; i < to && i < bytes; i++)
            if (raw[i]) return false;
        return true;
    };
    if (!p.q_ptr || !p.k_ptr || !p.v_ptr || !p.o_ptr) return declined(who, "null operand");
    if (p.oaccum_ptr || p.p_ptr || p.softmax_lseaccum_ptr)
        return declined(who, "split-k or dropout mask");
    if (p.seqlen_knew || p.rotary_dim) return declined(who, "kv cache or rotary");
    const bool causal = raw[ZLIFT_FLASH_IS_CAUSAL_BYTE] != 0;
    if (!causal && (p.window_size_left != -1 || p.window_size_right != -1))
        return declined(who, "local window");
    if (causal && p.window_size_right != 0) return declined(who, "local window");
    if (!zeroes(224, 372) || !zeroes(396, 440)) return declined(who, "a feature is set");
    if (p.p_dropout_in_uint8_t != 255) return declined(who, "dropout");
    if (p.p_dropout != 1.0f || p.rp_dropout != 1.0f) return declined(who, "dropout");
    if ((raw[ZLIFT_FLASH_IS_BF16_BYTE] != 0) != (elem == 1)) return declined(who, "dtype disagrees");
    if (p.b <= 0 || p.h <= 0 || p.seqlen_q <= 0 || p.seqlen_k <= 0) return declined(who, "empty");
    if (p.h_k <= 0 || p.h_h_k_ratio <= 0 || p.h != p.h_k * p.h_h_k_ratio)
        return declined(who, "head grouping");
    if (elem < 0 || elem > 2) return declined(who, "element type");
    zl::AttnDesc d{};
    d.q = p.q_ptr; d.k = p.k_ptr; d.v = p.v_ptr; d.o = p.o_ptr;
    d.lse = static_cast<float*>(p.softmax_lse_ptr);
    d.qb = p.q_batch_stride; d.qh = p.q_head_stride; d.qr = p.q_row_stride;
    d.kb = p.k_batch_stride; d.kh = p.k_head_stride; d.kr = p.k_row_stride;
    d.vb = p.v_batch_stride; d.vh = p.v_head_stride; d.vr = p.v_row_stride;
    d.ob = p.o_batch_stride; d.oh = p.o_head_stride; d.orr = p.o_row_stride;
    d.batches = p.b; d.heads = p.h; d.kv_ratio = p.h_h_k_ratio;
    d.sq = p.seqlen_q; d.sk = p.seqlen_k; d.d = p.d;
    d.scale = p.scale_softmax;
    d.causal = causal;
    d.diag = causal ? p.seqlen_k - p.seqlen_q : 0;   // bottom-right aligned
    d.elem = elem;
    if (pair_end > 0) {
        if (pair_begin < 0 || pair_end > (long long)p.b * p.h || pair_begin >= pair_end)
            return declined(who, "pair range");
        d.pair_begin = pair_begin;
        d.pair_end = pair_end;
    }
    return run(who, d, s);
}

}  // namespace zl

namespace {

// zblas/zblas_gpu.cpp:1424-1476
int fmha(const void* params, unsigned bytes, int elem, cudaStream_t s) {
    const char* who = "fmha";
    if (!params || bytes < sizeof(zlift_fmha_params)) return 1;
    zlift_fmha_params p;
    std::memcpy(&p, params, sizeof p);
    if (!p.query_ptr || !p.key_ptr || !p.value_ptr || !p.output_ptr)
        return declined(who, "null operand");
    if (p.seqstart_q_ptr || p.seqstart_k_ptr || p.seqlen_k_ptr) return declined(who, "ragged batch");
    if (p.custom_mask_type > 2) return declined(who, "unknown mask type");
    if (p.window_size != 0) return declined(who, "sliding window");
    if (p.use_dropout) return declined(who, "dropout");
    if (p.num_batches <= 0 || p.num_heads <= 0 || p.num_queries <= 0 || p.num_keys <= 0)
        return declined(who, "empty");
    if (p.head_dim != p.head_dim_value) return declined(who, "head_dim != head_dim_value");
    if (elem < 0 || elem > 2) return declined(who, "element type");
    zl::AttnDesc d{};
    d.q = p.query_ptr; d.k = p.key_ptr; d.v = p.value_ptr; d.o = p.output_ptr;
    d.lse = static_cast<float*>(p.logsumexp_ptr);
    d.qb = p.q_strideB; d.qh = p.q_strideH; d.qr = p.q_strideM;
    d.kb = p.k_strideB; d.kh = p.k_strideH; d.kr = p.k_strideM;
    d.vb = p.v_strideB; d.vh = p.v_strideH; d.vr = p.v_strideM;
    // output is [B, M, H, Kv] with row stride o_strideM (zblas_gpu.cpp:1448-1450)
    d.ob = (long long)p.num_queries * p.o_strideM;
    d.oh = p.head_dim_value;
    d.orr = p.o_strideM;
    // additive bias [b*strideB + h*strideH + query*strideM + key] of the input
    // type, added after scaling (zblas_gpu.cpp:963-966, :1451-1452)
    d.bias = p.attn_bias_ptr;
    d.bb = p.bias_strideB; d.bh = p.bias_strideH; d.br = p.bias_strideM;
    d.batches = p.num_batches; d.heads = p.num_heads; d.kv_ratio = 1;
    d.sq = p.num_queries; d.sk = p.num_keys; d.d = p.head_dim;
    d.scale = p.scale;
    d.causal = p.custom_mask_type != 0;
    d.diag = p.custom_mask_type == 2 ? p.num_keys - p.num_queries : 0;
    d.elem = elem;
    return run(who, d, s);
}

}  // namespace

extern "C" {

int zblas_gpu_flash_f16(const void* params, unsigned bytes, int elem) {
    return zl::flash_entry(params, bytes, elem, g_attn_stream, 0, 0);
}

int zblas_gpu_fmha_f16(const void* params, unsigned bytes, int elem) {
    return fmha(params, bytes, elem, g_attn_stream);
}

void zblas_attention_set_stream(void* stream) {
    g_attn_stream = static_cast<cudaStream_t>(stream);
}

void* zblas_attention_get_stream(void) { return g_attn_stream; }

int zlift_flash_fwd(const void* params, unsigned bytes, int elem, void* stream) {
    return zl::flash_entry(params, bytes, elem, static_cast<cudaStream_t>(stream), 0, 0);
}

int zlift_fmha_fwd(const void* params, unsigned bytes, int elem, void* stream) {
    return fmha(params, bytes, elem, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
