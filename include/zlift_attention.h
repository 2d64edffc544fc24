/*
 * zlift_attention.h -- fused-attention forward entry points.
 *
 * The reference answers attention inside its BLAS shim: the ZLUDA driver's
 * kernel-launch interception hands over the raw parameter block of an
 * intercepted FlashAttention-2 or xformers (cutlass FMHA) forward kernel
 * (zblas/zblas_gpu.cpp:1424-1535).  These declarations keep those two
 * entry points, their argument meaning and their parameter-block layouts,
 * and add an explicit-stream variant.  Exported by libcublas.so.13 and
 * re-exported by libcudnn.so.9.
 *
 * Return value of every entry: 0 = done (enqueued on the stream),
 * 1 = declined (the block asks for something this kernel does not do; the
 * caller must run the original kernel), as in the reference.
 *
 * Output: O in the input type, and -- new relative to the reference, which
 * never writes it -- the fp32 natural-log log-sum-exp of every query row
 * when the block carries an LSE pointer, laid out [batch][head][query].
 */
#ifndef ZLIFT_ATTENTION_H
#define ZLIFT_ATTENTION_H

#include <stddef.h>
#include <stdint.h>


#ifndef ZLIFT_API
#define ZLIFT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* FlashAttention-2 forward parameter block.  Field order and offsets are
 * the ones the reference pins (zblas/zblas_gpu.cpp:755-784); 448 bytes are
 * passed, bytes 440/441 carry is_bf16/is_causal.  Strides in elements. */
typedef struct zlift_flash_params {
    void *q_ptr, *k_ptr, *v_ptr;                                     /*   0 */
    long long q_batch_stride, k_batch_stride, v_batch_stride;        /*  24 */
    long long q_row_stride, k_row_stride, v_row_stride;              /*  48 */
    long long q_head_stride, k_head_stride, v_head_stride;           /*  72 */
    int h, h_k, h_h_k_ratio;                                         /*  96 */
    void *o_ptr, *oaccum_ptr;                                        /* 112 */
    long long o_batch_stride, o_row_stride, o_head_stride;           /* 128 */
    void *p_ptr;                                                     /* 152 */
    void *softmax_lse_ptr, *softmax_lseaccum_ptr;                    /* 160 */
    int b, seqlen_q, seqlen_k, seqlen_knew, d;                       /* 176 */
    int seqlen_q_rounded, seqlen_k_rounded, d_rounded;               /* 196 */
    int rotary_dim, total_q;                                         /* 208 */
    float scale_softmax, scale_softmax_log2;                         /* 216 */
    unsigned char opaque[148];                                       /* 224 */
    float p_dropout;                                                 /* 372 */
    unsigned char p_dropout_in_uint8_t;                              /* 376 */
    float rp_dropout;                                                /* 380 */
    float scale_softmax_rp_dropout;                                  /* 384 */
    int window_size_left, window_size_right;                         /* 388 */
} zlift_flash_params;

#define ZLIFT_FLASH_PARAMS_BYTES 448
#define ZLIFT_FLASH_IS_BF16_BYTE 440
#define ZLIFT_FLASH_IS_CAUSAL_BYTE 441

/* xformers cutlass FMHA forward parameter block (zblas/zblas_gpu.cpp:695-739).
 * custom_mask_type: 0 none, 1 causal from the top-left, 2 causal from the
 * bottom-right. */
typedef struct zlift_fmha_params {
    const void *query_ptr, *key_ptr, *value_ptr;                     /*   0 */
    const void *attn_bias_ptr;                                       /*  24 */
    const void *seqstart_q_ptr, *seqstart_k_ptr, *seqlen_k_ptr;      /*  32 */
    unsigned causal_diagonal_offset;                                 /*  56 */
    void *output_ptr, *output_accum_ptr, *logsumexp_ptr;             /*  64 */
    int window_size;                                                 /*  88 */
    float scale;                                                     /*  92 */
    int head_dim, head_dim_value, num_queries, num_keys;             /*  96 */
    int num_keys_absolute;                                           /* 112 */
    unsigned char custom_mask_type;                                  /* 116 */
    int q_strideM, k_strideM, v_strideM, bias_strideM, o_strideM;    /* 120 */
    int q_strideH, k_strideH, v_strideH;                             /* 140 */
    long long bias_strideH;                                          /* 152 */
    long long q_strideB, k_strideB, v_strideB, bias_strideB;         /* 160 */
    int num_batches, num_heads;                                      /* 192 */
    unsigned char use_dropout;                 /* 200; a C++ bool there */
} zlift_fmha_params;

/* elem: 0 = fp16, 1 = bf16, 2 = fp32 (fp32 is declined by this library). */

/* FlashAttention-2 forward.  Replaces zblas/zblas_gpu.cpp:1477-1535.
 * Runs on the stream set by zblas_attention_set_stream (default: the
 * legacy default stream). */
ZLIFT_API int zblas_gpu_flash_f16(const void *params, unsigned bytes, int elem);

/* xformers FMHA forward.  Replaces zblas/zblas_gpu.cpp:1424-1476.  Unlike
 * the reference, a block that asks for logsumexp is served (not declined). */
ZLIFT_API int zblas_gpu_fmha_f16(const void *params, unsigned bytes, int elem);

/* Stream for the two calls above (no reference counterpart: the reference
 * runs synchronously on its own queue, zblas_gpu.cpp:184-201). */
ZLIFT_API void zblas_attention_set_stream(void *stream);
ZLIFT_API void *zblas_attention_get_stream(void);

/* Same as zblas_gpu_flash_f16 / zblas_gpu_fmha_f16 on an explicit stream
 * (no reference counterpart). */
ZLIFT_API int zlift_flash_fwd(const void *params, unsigned bytes, int elem, void *stream);
ZLIFT_API int zlift_fmha_fwd(const void *params, unsigned bytes, int elem, void *stream);

#ifdef __cplusplus
}
#endif
#endif
