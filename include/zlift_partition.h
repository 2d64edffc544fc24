/*
 * zlift_partition.h -- the multi-GPU partition layer (no reference
 * counterpart: the reference is one device per process and has no
 * collective, zlift/src/run.rs:55-63).
 *
 * One process (or thread) per GPU.  Each rank calls the same per-GPU
 * kernels as the single-GPU entry points on its shard:
 *   - strided-batched GEMM: contiguous ranges of the batch;
 *   - attention: contiguous ranges of (batch, head) pairs, batch-major;
 *   - a large GEMM: contiguous ranges of C's columns (N-split), then one
 *     NCCL all-gather of the column blocks over NVLink.
 * The NCCL library is found at run time (the copy already loaded in the
 * process, else libnccl.so.2 on the loader path, else $ZLIFT_NCCL_LIB).
 *
 * Status returns: 0 success; 1 not available / bad argument; cuBLAS-style
 * statuses (7, 13, 15) from the GEMM calls; 100 + ncclResult_t for NCCL
 * failures; 200 when a bounded wait on a collective timed out (the
 * communicator is aborted).
 */
#ifndef ZLIFT_PARTITION_H
#define ZLIFT_PARTITION_H

#include <stddef.h>

#ifndef ZLIFT_API
#define ZLIFT_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Balanced contiguous split of `total` units over `parts` ranks, in
 * multiples of `align` units (the last rank takes the remainder).  Writes
 * [begin, end) of rank `index`.  Returns 1 on bad arguments. */
ZLIFT_API int zlift_part_range(long long total, int parts, int index, long long align,
                               long long *begin, long long *end);

/* NCCL communicator lifetime.  `id` is NCCL's 128-byte unique id: rank 0
 * creates it, the caller distributes it (any channel), every rank inits. */
ZLIFT_API int zlift_part_unique_id(void *id128);
ZLIFT_API int zlift_part_comm_init(void **comm, int nranks, int rank, const void *id128);
ZLIFT_API int zlift_part_comm_destroy(void *comm);

/* Waits until `stream` has drained, polling NCCL's asynchronous error;
 * after `timeout_ms` the communicator is aborted and 200 returned. */
ZLIFT_API int zlift_part_comm_wait(void *comm, void *stream, int timeout_ms);

/* Strided-batched GEMM restricted to batches [batch_begin, batch_end) of
 * the full problem (same arguments as cublasGemmStridedBatchedEx). */
ZLIFT_API int zlift_part_gemm_strided_batched_ex(
    void *handle, long long batch_begin, long long batch_end, int transa, int transb,
    int m, int n, int k, const void *alpha, const void *A, int Atype, int lda,
    long long strideA, const void *B, int Btype, int ldb, long long strideB,
    const void *beta, void *C, int Ctype, int ldc, long long strideC, int computeType);

/* N-split GEMM with all-gather.  Rank r of `nranks` owns columns
 * [n0, n1) = zlift_part_range(n, nranks, r, 128) of C.  `B_block` is that
 * rank's column block of op(B) (transb = N: k x (n1-n0), leading dim ldb).
 * `C` is the full m x n output (leading dimension m, contiguous); the rank
 * computes columns [n0, n1) into it and the all-gather fills the rest.
 * The handle's stream carries both the GEMM and the collective. */
ZLIFT_API int zlift_part_gemm_ex_nsplit(
    void *handle, void *comm, int nranks, int rank, int transa, int transb, int m, int n,
    int k, const void *alpha, const void *A, int Atype, int lda, const void *B_block,
    int Btype, int ldb, const void *beta, void *C, int Ctype, int computeType);

/* Attention forward restricted to (batch, head) pairs [pair_begin,
 * pair_end) in batch-major order, on `stream` (parameter block as for
 * zlift_flash_fwd).  0 done, 1 declined, 2 launch failure. */
ZLIFT_API int zlift_part_flash_fwd(const void *params, unsigned bytes, int elem,
                                   long long pair_begin, long long pair_end, void *stream);

#ifdef __cplusplus
}
#endif
#endif
