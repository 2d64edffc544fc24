"""Multi-GPU partition layer on real GPUs (skipped with fewer than 2).

One process per GPU (spawned here), NCCL communicator created by the
library (zlift_part_unique_id / zlift_part_comm_init; the id travels over a
gloo process group):
  - int8 N-split GEMM + all-gather, with the gather after the GEMM,
    overlapped with it sub-block by sub-block (NCCL), and by peer stores into
    a registered C (three steps in a row): every rank's gathered C equals
    the single-GPU product bit for bit;
  - flash forward split by (batch, head) pairs: each rank's pairs equal the
    single-GPU result bit for bit (same kernel, same tiles).
"""
import os
import socket

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _ngpus():
    import torch
    return torch.cuda.device_count() if torch.cuda.is_available() else 0


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out):
    import sys
    sys.path.insert(0, ROOT)
    from datetime import timedelta
    import torch
    import torch.distributed as dist
    import zlift_b200
    from zlift_b200 import blas, partition
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    comm = None
    try:
        box = [partition.Comm.unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        comm = partition.Comm(world, rank, box[0])
        stream = torch.cuda.current_stream()
        h = blas.Handle(stream)
        # ---- int8 N-split ----
        M, K, N = 512, 1024, 4096
        g = torch.Generator(device="cuda").manual_seed(11)
        A = torch.randint(-127, 128, (M, K), generator=g, device="cuda", dtype=torch.int8)
        Bfull = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
        n0, n1 = partition.shard_range(N, world, rank, 128)
        Bblk = Bfull[n0:n1].contiguous()
        C = torch.full((N, M), -1, dtype=torch.int32, device="cuda")
        st = partition.gemm_ex_nsplit(h, comm, world, rank, 1, 0, M, N, K, 1, A, 3, K, Bblk, 3,
                                      K, 0, C, 10, 72)
        assert st == 0, st
        assert comm.wait(stream, 30000) == 0
        ref = torch.empty_like(C)
        assert h.gemm_ex(1, 0, M, N, K, 1, A, 3, K, Bfull, 3, K, 0, ref, 10, M, compute=72) == 0
        torch.cuda.synchronize()
        ok_gemm = bool(torch.equal(C, ref))
        # ---- int8 N-split with the gather overlapped, 4 sub-blocks ----
        SB = 4
        cols = [partition.nsplit_cols(N, world, rank, SB, s) for s in range(SB)]
        Bcols = torch.cat([Bfull[b:e] for b, e in cols]).contiguous()
        C2 = torch.full((N, M), -1, dtype=torch.int32, device="cuda")
        st = partition.gemm_ex_nsplit_overlap(h, comm, world, rank, SB, 1, 0, M, N, K, 1, A, 3,
                                              K, Bcols, 3, K, 0, C2, 10, 72)
        assert st == 0, st
        assert comm.wait(stream, 30000) == 0
        torch.cuda.synchronize()
        ok_gemm = ok_gemm and bool(torch.equal(C2, ref))
        # ---- the same, gathered by peer stores into a registered C, three
        # steps in a row with different B (epochs advance, C is reused) ----
        C3 = torch.full((N, M), -1, dtype=torch.int32, device="cuda")
        assert comm.register_peer_buffer(C3, C3.numel() * 4) == 0
        for step in range(3):
            Bs = torch.randint(-127, 128, (N, K), generator=g, device="cuda", dtype=torch.int8)
            Bc = torch.cat([Bs[b:e] for b, e in cols]).contiguous()
            st = partition.gemm_ex_nsplit_overlap(h, comm, world, rank, SB, 1, 0, M, N, K, 1, A,
                                                  3, K, Bc, 3, K, 0, C3, 10, 72)
            assert st == 0, st
            ref3 = torch.empty_like(C3)
            assert h.gemm_ex(1, 0, M, N, K, 1, A, 3, K, Bs, 3, K, 0, ref3, 10, M,
                             compute=72) == 0
            torch.cuda.synchronize()
            ok_gemm = ok_gemm and bool(torch.equal(C3, ref3))
        torch.cuda.synchronize()
        dist.barrier()
        assert comm.unregister_peer_buffer(C3) == 0
        # ---- attention split by (batch, head) ----
        Bq, S, H, D = 2, 512, 4, 128
        q = torch.randn(Bq, S, H, D, generator=g, device="cuda").bfloat16()
        k = torch.randn(Bq, S, H, D, generator=g, device="cuda").bfloat16()
        v = torch.randn(Bq, S, H, D, generator=g, device="cuda").bfloat16()
        o_full = torch.empty_like(q)
        assert zlift_b200.flash_forward(q, k, v, o_full, None, causal=True) == 0
        o_part = torch.zeros_like(q)
        blk = zlift_b200.attention.flash_block(q, k, v, o_part, None, causal=True)
        p0, p1 = partition.shard_range(Bq * H, world, rank)
        assert partition.flash_pairs(blk, 1, p0, p1, stream) == 0
        torch.cuda.synchronize()
        ok_attn = True
        for pr in range(p0, p1):
            b, hh = divmod(pr, H)
            ok_attn &= bool(torch.equal(o_part[b, :, hh], o_full[b, :, hh]))
        out[rank] = (ok_gemm, ok_attn, blas.device_error())
        h.close()
    finally:
        if comm is not None:
            comm.close()
        dist.destroy_process_group()


@pytest.mark.skipif(_ngpus() < 2, reason="needs 2 GPUs")
def test_partition_two_gpus():
    import torch.multiprocessing as mp
    world = 2
    mgr = mp.get_context("spawn").Manager()
    out = mgr.dict()
    mp.spawn(_worker, args=(world, _port(), out), nprocs=world, join=True)
    assert dict(out) == {r: (True, True, 0) for r in range(world)}
