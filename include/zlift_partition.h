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

/* Column ownership of the overlapped N-split: the n columns form
 * `sub_blocks` super-blocks of n / sub_blocks columns each, and within each
 * super-block rank r owns the r-th of nranks equal pieces of
 * w = n / (sub_blocks * nranks) columns.  Writes the global columns
 * [begin, end) of rank `rank`'s sub-block `s`.  Returns 1 on bad arguments
 * or when w is not a whole number. */
ZLIFT_API int zlift_part_nsplit_cols(long long n, int nranks, int rank, int sub_blocks, int s,
                                     long long *begin, long long *end);

/* N-split GEMM whose all-gather overlaps the GEMM.  Extends cublasGemmEx
 * (zblas/zblas.c:357-391) across GPUs, like zlift_part_gemm_ex_nsplit, but
 * with the interleaved column ownership of zlift_part_nsplit_cols:
 * `B_cols` holds this rank's sub-blocks of op(B) back to back (sub-block s
 * = the w columns zlift_part_nsplit_cols gives for s; transb = N:
 * k x (sub_blocks * w), leading dim ldb).  The GEMM of each sub-block runs
 * on the handle's stream (using all SMs but ZLIFT_PART_COMM_SMS, default
 * 16, so NCCL's kernels run next to it); each super-block's in-place
 * ncclAllGather runs on a second stream of the communicator as soon as
 * this rank's GEMM of it is done, overlapping the next sub-block's GEMM.
 * The handle's stream waits for the last gather: C (m x n, leading dim m)
 * is complete there, as with zlift_part_gemm_ex_nsplit.  Every rank calls
 * it with the same sizes and sub_blocks. */
ZLIFT_API int zlift_part_gemm_ex_nsplit_overlap(
    void *handle, void *comm, int nranks, int rank, int sub_blocks, int transa, int transb,
    int m, int n, int k, const void *alpha, const void *A, int Atype, int lda,
    const void *B_cols, int Btype, int ldb, const void *beta, void *C, int Ctype,
    int computeType);

/* Maps a full-size output buffer C (`bytes` long, device memory of this
 * rank) into every rank's address space (CUDA IPC, handles exchanged through
 * the communicator) and gives it a flag array.  Collective: every rank calls
 * it with its own C, the same `bytes`, before the first step that uses it;
 * the buffer ends up registered on every rank or on none (the ranks agree on
 * the first nonzero status).  A C already registered with this communicator
 * returns 0 at once, without the exchange, so every rank must make the same
 * calls in the same order.  Afterwards zlift_part_gemm_ex_nsplit_overlap on
 * this C gathers each sub-block straight into the peers' C instead of
 * through ncclAllGather: by copy-engine copies, one stream per peer
 * (default), or by a store kernel next to the GEMM of the following
 * sub-block (ZLIFT_PART_GATHER=sm).  READY / DONE flags between the ranks
 * order it, every wait bounded by the library's wait limit (a timeout is
 * reported by zlift_device_error; a rank whose call failed part-way sends no
 * DONE, so its peers time out rather than read partial columns).  Up to 8
 * ranks.  Each exchange step waits at most 120 s for the other ranks, then
 * aborts the communicator (200).  0 success, 1 bad arguments, 13 a CUDA call
 * failed (on this rank or, reported through the agreement, on another);
 * 100 + ncclResult_t (a collective failed) and 200 (a rank did not arrive)
 * mean this rank's communicator has been aborted: it must not be used or
 * destroyed afterwards. */
ZLIFT_API int zlift_part_register_peer_buffer(void *comm, int nranks, int rank, void *C,
                                             size_t bytes);
/* Unmaps a registered C (after every rank's last use of it; waits for the
 * device).  Also done for all of a communicator's buffers by
 * zlift_part_comm_destroy.  1 if C was not registered. */
ZLIFT_API int zlift_part_unregister_peer_buffer(void *comm, void *C);

/* Attention forward restricted to (batch, head) pairs [pair_begin,
 * pair_end) in batch-major order, on `stream` (parameter block as for
 * zlift_flash_fwd).  0 done, 1 declined, 2 launch failure. */
ZLIFT_API int zlift_part_flash_fwd(const void *params, unsigned bytes, int elem,
                                   long long pair_begin, long long pair_end, void *stream);

#ifdef __cplusplus
}
#endif
#endif
