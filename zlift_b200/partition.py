"""Python side of the partition layer (include/zlift_partition.h).

The shard arithmetic and the collective live in libcublas.so.13; this
module only forwards to it.  `Comm` wraps an NCCL communicator created by
the library; its 128-byte unique id travels over whatever channel the
caller has (torch.distributed here).
"""
from __future__ import annotations

import ctypes

from . import load


def shard_range(total: int, parts: int, index: int, align: int = 1) -> tuple[int, int]:
    """[begin, end) of rank `index` of `parts` over `total` units, in
    multiples of `align` (zlift_part_range)."""
    b, e = ctypes.c_longlong(), ctypes.c_longlong()
    rc = load().zlift_part_range(total, parts, index, align, ctypes.byref(b), ctypes.byref(e))
    if rc:
        raise ValueError(f"zlift_part_range({total}, {parts}, {index}, {align}) -> {rc}")
    return b.value, e.value


def flash_pairs(block, elem: int, pair_begin: int, pair_end: int, stream=None) -> int:
    """Flash forward over (batch, head) pairs [pair_begin, pair_end)."""
    s = 0 if stream is None else int(getattr(stream, "cuda_stream", stream))
    return load().zlift_part_flash_fwd(ctypes.byref(block), ctypes.sizeof(block), elem,
                                       pair_begin, pair_end, s)


class PeerLost(RuntimeError):
    """A rank did not announce the next step in time (it left the job)."""


class Heartbeat:
    """Host-side liveness check between steps of a multi-GPU job.

    Before launching step `i`, every rank calls ``beat(i)``: it publishes
    ``hb/<i>/<rank>`` in the job's key-value store and waits, up to
    `timeout_s`, for every other rank's key of the same step.  A rank that
    left the job between steps is seen here, on the host, before any kernel
    or collective of step `i` is launched -- so no GPU ever waits on a peer
    that is gone.  Raises PeerLost (with the missing ranks) on expiry.

    The store is any torch.distributed Store (TCPStore, FileStore, ...).
    """

    def __init__(self, store, world: int, rank: int, timeout_s: float = 5.0):
        self.store, self.world, self.rank = store, world, rank
        self.timeout_s = timeout_s

    def beat(self, step: int) -> None:
        from datetime import timedelta
        self.store.set(f"hb/{step}/{self.rank}", "1")
        others = [f"hb/{step}/{r}" for r in range(self.world) if r != self.rank]
        if not others:
            return
        try:
            self.store.wait(others, timedelta(seconds=self.timeout_s))
        except Exception as e:            # store timeout or a closed store
            missing = []
            for r in range(self.world):
                if r == self.rank:
                    continue
                try:
                    if not self.store.check([f"hb/{step}/{r}"]):
                        missing.append(r)
                except Exception:
                    missing.append(r)
            raise PeerLost(f"step {step}: no heartbeat from rank(s) {missing or '?'}") from e


class Comm:
    """NCCL communicator of the partition layer."""

    def __init__(self, nranks: int, rank: int, unique_id: bytes):
        self.lib = load()
        c = ctypes.c_void_p()
        buf = ctypes.create_string_buffer(unique_id, 128)
        rc = self.lib.zlift_part_comm_init(ctypes.byref(c), nranks, rank, buf)
        if rc:
            raise RuntimeError(f"zlift_part_comm_init -> {rc}")
        self.c, self.nranks, self.rank = c, nranks, rank

    @staticmethod
    def unique_id() -> bytes:
        buf = ctypes.create_string_buffer(128)
        rc = load().zlift_part_unique_id(buf)
        if rc:
            raise RuntimeError(f"zlift_part_unique_id -> {rc}")
        return buf.raw

    def wait(self, stream, timeout_ms: int = 10000) -> int:
        """Waits for `stream` with a deadline (zlift_part_comm_wait): 0 once
        the stream's work is done; 200 past the deadline and 100 + NCCL's
        code on an asynchronous NCCL error -- the library has then aborted
        the communicator, which this object drops."""
        s = int(getattr(stream, "cuda_stream", stream or 0))
        rc = self.lib.zlift_part_comm_wait(self.c, s, timeout_ms)
        if rc >= 100:
            self.c = None
        return rc

    def register_peer_buffer(self, C, nbytes: int) -> int:
        """Collective: maps C into every rank (zlift_part_register_peer_buffer),
        so the overlapped N-split gathers into it by peer stores.  A result of
        100 or more means the library aborted the communicator (a collective
        failed, or a rank did not arrive); this object then drops it."""
        from .blas import _ptr
        rc = self.lib.zlift_part_register_peer_buffer(self.c, self.nranks, self.rank, _ptr(C),
                                                      nbytes)
        if rc >= 100:
            self.c = None
        return rc

    def unregister_peer_buffer(self, C) -> int:
        from .blas import _ptr
        return self.lib.zlift_part_unregister_peer_buffer(self.c, _ptr(C))

    def close(self):
        if self.c:
            self.lib.zlift_part_comm_destroy(self.c)
            self.c = None


def gemm_ex_nsplit(handle, comm, nranks, rank, transa, transb, m, n, k, alpha, A, Atype, lda,
                   B_block, Btype, ldb, beta, C, Ctype, compute) -> int:
    """N-split GEMM + all-gather (zlift_part_gemm_ex_nsplit)."""
    from .blas import COMPUTE_32I, R_32I, _ptr
    integer = compute in (COMPUTE_32I, R_32I)
    al = ctypes.c_int32(int(alpha)) if integer else ctypes.c_float(float(alpha))
    be = ctypes.c_int32(int(beta)) if integer else ctypes.c_float(float(beta))
    return load().zlift_part_gemm_ex_nsplit(
        handle.h, comm.c if comm is not None else None, nranks, rank, transa, transb, m, n, k,
        ctypes.byref(al), _ptr(A), Atype, lda, _ptr(B_block), Btype, ldb, ctypes.byref(be),
        _ptr(C), Ctype, compute)


def gemm_strided_batched_range(handle, batch_begin, batch_end, transa, transb, m, n, k, alpha,
                               A, Atype, lda, sA, B, Btype, ldb, sB, beta, C, Ctype, ldc, sC,
                               compute) -> int:
    from .blas import COMPUTE_32I, R_32I, _ptr
    integer = compute in (COMPUTE_32I, R_32I)
    al = ctypes.c_int32(int(alpha)) if integer else ctypes.c_float(float(alpha))
    be = ctypes.c_int32(int(beta)) if integer else ctypes.c_float(float(beta))
    return load().zlift_part_gemm_strided_batched_ex(
        handle.h, batch_begin, batch_end, transa, transb, m, n, k, ctypes.byref(al), _ptr(A),
        Atype, lda, sA, _ptr(B), Btype, ldb, sB, ctypes.byref(be), _ptr(C), Ctype, ldc, sC,
        compute)


def nsplit_cols(n: int, nranks: int, rank: int, sub_blocks: int, s: int) -> tuple[int, int]:
    """Global columns [begin, end) of `rank`'s sub-block `s` in the
    overlapped N-split (zlift_part_nsplit_cols)."""
    b, e = ctypes.c_longlong(), ctypes.c_longlong()
    rc = load().zlift_part_nsplit_cols(n, nranks, rank, sub_blocks, s, ctypes.byref(b),
                                       ctypes.byref(e))
    if rc:
        raise ValueError(f"zlift_part_nsplit_cols({n}, {nranks}, {rank}, {sub_blocks}, {s})")
    return b.value, e.value


def gemm_ex_nsplit_overlap(handle, comm, nranks, rank, sub_blocks, transa, transb, m, n, k,
                           alpha, A, Atype, lda, B_cols, Btype, ldb, beta, C, Ctype,
                           compute) -> int:
    """N-split GEMM with its all-gather overlapped, sub-block by sub-block
    (zlift_part_gemm_ex_nsplit_overlap)."""
    from .blas import COMPUTE_32I, R_32I, _ptr
    integer = compute in (COMPUTE_32I, R_32I)
    al = ctypes.c_int32(int(alpha)) if integer else ctypes.c_float(float(alpha))
    be = ctypes.c_int32(int(beta)) if integer else ctypes.c_float(float(beta))
    return load().zlift_part_gemm_ex_nsplit_overlap(
        handle.h, comm.c if comm is not None else None, nranks, rank, sub_blocks, transa,
        transb, m, n, k, ctypes.byref(al), _ptr(A), Atype, lda, _ptr(B_cols), Btype, ldb,
        ctypes.byref(be), _ptr(C), Ctype, compute)
