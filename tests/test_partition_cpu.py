"""CPU: the partition layer's host logic.

- zlift_part_range (the shard planner) covers every unit exactly once, in
  order, aligned, for the batch, (batch, head) and column splits;
- a world_size-2 gloo job runs the N-split GEMM's data flow on the CPU:
  each rank computes its column block of C with the oracle and an
  all-gather in rank order reassembles exactly the full product -- the
  same block order the library's NCCL all-gather produces.
"""
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("total,parts,align", [
    (256, 1, 1), (256, 2, 1), (256, 3, 1), (256, 8, 1), (5, 8, 1),
    (14336, 8, 128), (14336, 3, 128), (1000, 4, 128), (0, 4, 1), (256, 7, 16),
])
def test_shard_ranges_partition_exactly(built_lib, total, parts, align):
    from zlift_b200 import partition
    prev = 0
    sizes = []
    for r in range(parts):
        b, e = partition.shard_range(total, parts, r, align)
        assert b == prev and e >= b
        if e < total:
            assert e % align == 0
        prev = e
        sizes.append(e - b)
    assert prev == total
    units = [(s + align - 1) // align for s in sizes]
    assert max(units) - min(units) <= 1 or total < parts * align


def test_shard_range_rejects_bad_arguments(built_lib):
    from zlift_b200 import partition
    for args in ((10, 0, 0, 1), (10, 2, 2, 1), (10, 2, -1, 1), (-1, 2, 0, 1), (10, 2, 0, 0)):
        with pytest.raises(ValueError):
            partition.shard_range(*args)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _nsplit_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from oracle import oracle
    from zlift_b200 import inputs, partition
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        M, K, N = 64, 96, 384
        A = inputs.int8(1, K * M)              # op(A) = A^T, stored K x M
        Bfull = inputs.int8(2, K * N)          # K x N column-major
        n0, n1 = partition.shard_range(N, world, rank, 128)
        Bblk = Bfull[n0 * K:n1 * K].copy()
        C = np.zeros(M * (n1 - n0), np.int32)
        assert oracle.gemm_ex(1, 0, M, n1 - n0, K, 1, A, 3, K, Bblk, 3, K, 0, C, 10, M,
                              72) == 0
        blocks = [torch.zeros(M * 128, dtype=torch.int32) for _ in range(world)]
        dist.all_gather(blocks, torch.from_numpy(C))
        full = torch.cat(blocks).numpy()
        want = np.zeros(M * N, np.int32)
        oracle.gemm_ex(1, 0, M, N, K, 1, A, 3, K, Bfull, 3, K, 0, want, 10, M, 72)
        out[rank] = bool(np.array_equal(full, want))
    finally:
        dist.destroy_process_group()


def test_nsplit_allgather_assembles_full_product_gloo(built_lib, oracle_lib):
    import torch.multiprocessing as mp
    world = 3
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    ctx = mp.spawn(_nsplit_worker, args=(world, port, out), nprocs=world, join=True)
    assert dict(out) == {r: True for r in range(world)}


def _pair_worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    import torch
    import torch.distributed as dist
    from zlift_b200 import partition
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, H = 8, 32
        b, e = partition.shard_range(B * H, world, rank)
        mine = torch.zeros(B * H, dtype=torch.int32)
        mine[b:e] = 1
        dist.all_reduce(mine)
        out[rank] = bool(torch.all(mine == 1))
    finally:
        dist.destroy_process_group()


def test_pair_split_covers_every_batch_head_once_gloo(built_lib):
    import torch.multiprocessing as mp
    world = 2
    port = _free_port()
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_pair_worker, args=(world, port, out), nprocs=world, join=True)
    assert dict(out) == {0: True, 1: True}


@pytest.mark.parametrize("n,nranks,sb", [(14336, 2, 4), (14336, 4, 4), (14336, 8, 2), (4096, 2, 4),
                                         (384, 3, 1), (64, 8, 8)])
def test_nsplit_cols_cover_every_column_once(built_lib, n, nranks, sb):
    """Overlapped N-split ownership: super-block s holds every rank's
    sub-block s in rank order, so each super-block is one in-place
    all-gather, and the union over ranks and sub-blocks is every column."""
    from zlift_b200 import partition
    owner = np.full(n, -1)
    for s in range(sb):
        prev = s * (n // sb)
        for r in range(nranks):
            b, e = partition.nsplit_cols(n, nranks, r, sb, s)
            assert b == prev and e - b == n // (sb * nranks)
            assert np.all(owner[b:e] == -1)
            owner[b:e] = r
            prev = e
        assert prev == (s + 1) * (n // sb)
    assert np.all(owner >= 0)


def test_nsplit_cols_rejects_uneven(built_lib):
    from zlift_b200 import partition
    for args in ((100, 3, 1, 1, 0), (14338, 8, 0, 4, 0), (10, 2, 2, 1, 0), (10, 2, 0, 1, 1)):
        with pytest.raises(ValueError):
            partition.nsplit_cols(*args)
