/*
 * cudnn_attention.c -- libcudnn.so.9: the attention entry points under the
 * cuDNN library name.  zLift ships its DNN shim as libcudnn.so.9
 * (zdnn/build.sh:15-17) and the task places the fused attention forward
 * there; the kernels themselves live in libcublas.so.13 (where the
 * reference's attention code sits, zblas/zblas_gpu.cpp:1424-1535), so
 * each entry here forwards to that library.
 */
#include "zlift_attention.h"

int zblas_gpu_flash_f16(const void *params, unsigned bytes, int elem) {
    return zlift_flash_fwd(params, bytes, elem, zblas_attention_get_stream());
}

int zblas_gpu_fmha_f16(const void *params, unsigned bytes, int elem) {
    return zlift_fmha_fwd(params, bytes, elem, zblas_attention_get_stream());
}

/* cudnnGetVersion: the cuDNN 9 version number this library stands in for. */
size_t cudnnGetVersion(void) { return 90000; }
