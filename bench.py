"""Benchmark of the GEMM / fused-attention hot path (one JSON line on rank 0).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload all|gemm_f16|gemm_bf16_batched|gemm_i8|fmha|sgemm]

The default (`all`) measures every benchmark configuration in one run and
prints one line: the headline keys (`value`, `roofline`, `e2e`, ...) are
those of gemm_f16, the configuration the metric is quoted on, and
`configs` holds one record of the same keys per configuration:

  sgemm              cublasSgemm_v2 fp32 M=N=K=1024 NN (3-product tf32);
                     N>1: replicas, one per GPU.
  gemm_f16           cublasGemmEx fp16 in / fp32 accumulate / fp16 out,
                     M=N=K=4096, transa=N transb=T, alpha=1 beta=0.5;
                     N>1: replicas, one per GPU.
  gemm_bf16_batched  cublasGemmStridedBatchedEx bf16, batch 256 of 512^3 NN,
                     alpha=1/sqrt(512), beta=0; N>1: batch split across GPUs
                     (zlift_part_gemm_strided_batched_ex), no collective.
  gemm_i8            cublasGemmEx int8 -> int32, M=2048 K=4096 N=14336, TN;
                     N>1: N-column split and a gather of C, in the form
                     measured fastest at that N: at N = 2 each column
                     sub-block is copied into the peer's C by the copy
                     engines while the next is computed (registered buffer,
                     zlift_part_gemm_ex_nsplit_overlap), above that one NCCL
                     all-gather after the GEMM (zlift_part_gemm_ex_nsplit);
                     the other form is reported too (gemm_i8_serialgather at
                     N = 2, gemm_i8_peercopy above), and the split without
                     any gather (gemm_i8_nogather).
  fmha               flash forward bf16 B=8 H=32 S=4096 D=128 causal, fp32
                     LSE; N>1: (batch, head) pairs split across GPUs
                     (zlift_part_flash_fwd), no collective.

A step is one call of the hot path over one batch of input already in HBM
(`value`).  Each configuration's timed region is exactly K steps between a
barrier and a device synchronisation on every rank, timed with CUDA events
on the launching stream and reduced with MAX over ranks; the region is
repeated (`repeats`) so that the clock sampler sees the GPU under load for
a while, and the median repeat is reported.  `e2e` repeats the step
through the same C ABI with pinned host buffers copied in and the result
copied out inside the timed region, every step: pipelined over two device
buffer slots (step i+1's upload on one copy stream while step i computes
and downloads on another; PCIe is full duplex), with the one-stream serial
figure reported beside it (`serial_ms_per_step`).  `cpu_baseline` (rank 0, N=1) and
`--impl reference` time the reference's own CPU implementation -- zblas.c
built from the reference sources (oracle/_ref) where the reference has a
CPU path, the oracle's C restatement where it has none (int8, attention) --
on this host's cores, on a bounded sample of the same workload.
"""
from __future__ import annotations

import os
import sys

# Thread counts of the host BLAS / OpenMP must be fixed before numpy (and
# its OpenBLAS) load.  torchrun exports OMP_NUM_THREADS=1 to every rank; the
# CPU measurements (the reference arm, and the CPU baseline at N=1) use
# every core this process may run on.
_CORES = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
if any(a.endswith("reference") for a in sys.argv) or os.environ.get("WORLD_SIZE", "1") == "1":
    os.environ["OPENBLAS_NUM_THREADS"] = str(_CORES)
    os.environ["OMP_NUM_THREADS"] = str(_CORES)

import argparse  # noqa: E402
import json  # noqa: E402
import math  # noqa: E402
import statistics  # noqa: E402
import threading  # noqa: E402
import time  # noqa: E402

import numpy as np  # noqa: E402

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "GemmEx TFLOP/s (bf16/fp16/int8 TOPS) & FMHA fwd TFLOP/s vs tensor-core peak"
HEADLINE = "gemm_f16"
ORDER = ["sgemm", "gemm_f16", "gemm_bf16_batched", "gemm_i8", "fmha"]


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}, "fallback"


def traffic_from_profile(workload: str):
    """Per-launch DRAM bytes of the dominant kernel from the committed ncu
    summary (profiles/<workload>_traffic.txt, line 'dram_bytes_per_launch: N')."""
    p = os.path.join(ROOT, "profiles", f"{workload}_traffic.txt")
    if not os.path.exists(p):
        return None
    with open(p) as f:
        for line in f:
            if line.startswith("dram_bytes_per_launch:"):
                return float(line.split(":", 1)[1].split()[0])
    return None


# --------------------------------------------------------------------------
# clocks: NVML sampled on a thread for the whole run; each timed region
# summarises the samples taken inside it
# --------------------------------------------------------------------------

class ClockSampler:
    REASONS = {
        0x0000000000000004: "sw_power_cap",
        0x0000000000000008: "hw_slowdown",
        0x0000000000000020: "sw_thermal_slowdown",
        0x0000000000000040: "hw_thermal_slowdown",
        0x0000000000000080: "hw_power_brake_slowdown",
    }

    def __init__(self, index: int, period_s: float = 0.004):
        self.samples = []          # (time, sm MHz, reason names)
        self.max_mhz = None
        self.period = period_s
        self.ok = False
        try:
            import pynvml
            pynvml.nvmlInit()
            self.nv = pynvml
            self.h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
            self.ok = True
        except Exception:
            self.ok = False
        self._stop = threading.Event()
        self._t = None
        self.windows = []          # (t0, t1) of the timed regions

    def _run(self):
        while not self._stop.is_set():
            try:
                mhz = self.nv.nvmlDeviceGetClockInfo(self.h, self.nv.NVML_CLOCK_SM)
                r = self.nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                names = tuple(n for bit, n in self.REASONS.items() if r & bit)
                self.samples.append((time.perf_counter(), mhz, names))
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.ok and self._t is None:
            self._t = threading.Thread(target=self._run, daemon=True)
            self._t.start()

    def stop(self):
        self._stop.set()
        if self._t:
            self._t.join()
            self._t = None

    def summary(self, windows):
        sel = [s for s in self.samples if any(a <= s[0] <= b for a, b in windows)]
        reasons = sorted({n for s in sel for n in s[2]})
        if not sel:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": reasons,
                    "samples": 0}
        return {"sm_mhz": float(statistics.median(s[1] for s in sel)),
                "sm_max_mhz": self.max_mhz, "reasons": reasons, "samples": len(sel),
                "window_s": round(sum(b - a for a, b in windows), 3)}


# --------------------------------------------------------------------------
# workloads (our arm)
# --------------------------------------------------------------------------

def _gen(kind, shape, seed, device, scale=1.0):
    import torch
    g = torch.Generator(device=device).manual_seed(seed)
    if kind == "i8":
        return torch.randint(-127, 128, shape, generator=g, device=device, dtype=torch.int8)
    x = torch.randn(shape, generator=g, device=device, dtype=torch.float32) * scale
    return x.to({"f16": torch.float16, "bf16": torch.bfloat16, "f32": torch.float32}[kind])


class Workload:
    name = ""
    dtype = ""
    unit = "TFLOP/s"
    scaling = "weak"
    bound = "tensor"
    peak_scale = 1.0        # dense rate of this arithmetic / bf16 rate
    flops = 0.0             # per step, whole job
    kernel_flops = 0.0      # per launch of the dominant kernel (this rank)
    kernel_bytes = 0.0      # algorithmic bytes per launch of the dominant kernel
    launches_per_step = 1

    @staticmethod
    def config_for(world):
        return {}

    def config(self):
        return self.config_for(self.world)

    # e2e: two device buffer slots; step i uploads slot i % 2's inputs from
    # pinned host memory, runs the step on them and downloads its result
    def e2e_upload(self, slot):
        raise NotImplementedError

    def e2e_compute(self, slot):
        raise NotImplementedError

    def e2e_download(self, slot):
        raise NotImplementedError

    def close(self):
        pass


class GemmF16(Workload):
    """cublasGemmEx fp16, 4096^3, NT, alpha 1 beta 0.5; 3 rotating input sets
    (3 x 96 MiB > 126 MiB L2) so no step reads operands left in L2."""
    name, dtype = "gemm_f16", "f16"
    M = N = K = 4096

    @staticmethod
    def config_for(world):
        return {"workload": "cublasGemmEx fp16->fp16 (fp32 accumulate) M=N=K=4096 transa=N "
                            "transb=T alpha=1 beta=0.5", "m": 4096, "n": 4096, "k": 4096,
                "inputs": "A,B ~ N(0,1)/64, C ~ N(0,1) (seeded)",
                "l2": "3 rotating input sets of 96 MiB (> 126 MiB L2 between reuses)",
                "parallelism": f"replicas x{world}"}

    def __init__(self, h, dev, rank, world, stream):
        import torch
        self.h, self.world = h, world
        M, N, K = self.M, self.N, self.K
        self.sets = []
        for s in range(3):
            A = _gen("f16", (K, M), 10 + s, dev, 1.0 / 64)        # col-major M x K
            B = _gen("f16", (K, N), 20 + s, dev, 1.0 / 64)        # col-major N x K (op T)
            C = _gen("f16", (N, M), 30 + s, dev)                 # col-major M x N
            self.sets.append((A, B, C))
        self.flops = 2.0 * M * N * K * world
        self.kernel_flops = 2.0 * M * N * K
        self.kernel_bytes = 2.0 * (M * K + K * N + 2 * M * N)
        A, B, C = self.sets[0]
        self.hA, self.hB, self.hC = (t.cpu().pin_memory() for t in (A, B, C))
        self.hOut = [torch.empty_like(self.hC).pin_memory() for _ in range(2)]

    def step(self, i):
        A, B, C = self.sets[i % 3]
        st = self.h.gemm_ex(0, 1, self.M, self.N, self.K, 1.0, A, 2, self.M, B, 2, self.N,
                            0.5, C, 2, self.M)
        assert st == 0, st

    def e2e_upload(self, slot):
        for d, hsrc in zip(self.sets[slot], (self.hA, self.hB, self.hC)):
            d.copy_(hsrc, non_blocking=True)

    def e2e_compute(self, slot):
        self.step(slot)

    def e2e_download(self, slot):
        self.hOut[slot].copy_(self.sets[slot][2], non_blocking=True)

    def e2e_bytes(self):
        return 2 * (2 * self.M * self.K + self.M * self.N), 2 * self.M * self.N

    def library(self):
        """torch.addmm (cuBLAS) on the same shape and layout, same box."""
        import itertools
        import torch
        calls = []
        for A, B, C in self.sets:             # the same 3 rotating input sets
            a = A.view(self.K, self.M).t()    # M x K view of column-major A
            b = B.view(self.K, self.N)        # op(B) = B^T (N x K stored): K x N
            c = C.view(self.N, self.M).t()
            calls.append((a, b, c, torch.empty_like(c)))
        it = itertools.cycle(calls)

        def run():
            a, b, c, out = next(it)
            return torch.addmm(c, a, b, beta=0.5, alpha=1.0, out=out)
        return run, "torch.addmm fp16 (NVIDIA cuBLAS), same shape/layout/alpha/beta, 3 input sets"


class GemmBF16Batched(Workload):
    name, dtype, scaling, bound = "gemm_bf16_batched", "bf16", "strong", "hbm"
    BATCH, M, N, K = 256, 512, 512, 512

    @staticmethod
    def config_for(world):
        return {"workload": "cublasGemmStridedBatchedEx bf16->bf16 batch=256 M=N=K=512 NN "
                            "alpha=1/sqrt(512) beta=0", "batch": 256, "m": 512, "n": 512,
                "k": 512, "inputs": "A,B ~ N(0,1) (seeded)",
                "l2": "inputs (256 MiB) + output (128 MiB) larger than L2",
                "parallelism": f"batch-split x{world} (zlift_part_gemm_strided_batched_ex)"}

    def __init__(self, h, dev, rank, world, stream):
        import torch
        from zlift_b200 import partition
        self.h, self.world = h, world
        lo, hi = partition.shard_range(self.BATCH, world, rank)
        self.lo, self.hi = lo, hi
        M, N, K = self.M, self.N, self.K
        # each rank holds the whole batch's layout but touches only its range
        # (the partition entry offsets the pointers)
        self.A = _gen("bf16", (self.BATCH, K, M), 40, dev)
        self.B = _gen("bf16", (self.BATCH, N, K), 50, dev)
        self.C = torch.empty(self.BATCH, N, M, dtype=torch.bfloat16, device=dev)
        # the e2e pipeline's second buffer slot
        self.slots = [(self.A, self.B, self.C),
                      tuple(torch.empty_like(t) for t in (self.A, self.B, self.C))]
        nb = hi - lo
        self.flops = 2.0 * M * N * K * self.BATCH
        self.kernel_flops = 2.0 * M * N * K * nb
        self.kernel_bytes = 2.0 * (M * K + K * N + M * N) * nb
        self.hA = self.A[lo:hi].cpu().pin_memory()
        self.hB = self.B[lo:hi].cpu().pin_memory()
        self.hC = [torch.empty_like(self.C[lo:hi], device="cpu").pin_memory() for _ in range(2)]

    def _gemm(self, A, B, C):
        from zlift_b200 import partition
        M, N, K = self.M, self.N, self.K
        st = partition.gemm_strided_batched_range(
            self.h, self.lo, self.hi, 0, 0, M, N, K, 1.0 / math.sqrt(K), A, 14, M, M * K,
            B, 14, K, K * N, 0.0, C, 14, M, M * N, 68)
        assert st == 0, st

    def step(self, i):
        self._gemm(self.A, self.B, self.C)

    def e2e_upload(self, slot):
        A, B, _ = self.slots[slot]
        A[self.lo:self.hi].copy_(self.hA, non_blocking=True)
        B[self.lo:self.hi].copy_(self.hB, non_blocking=True)

    def e2e_compute(self, slot):
        self._gemm(*self.slots[slot])

    def e2e_download(self, slot):
        self.hC[slot].copy_(self.slots[slot][2][self.lo:self.hi], non_blocking=True)

    def e2e_bytes(self):
        nb = self.hi - self.lo
        return 2 * (self.M * self.K + self.K * self.N) * nb, 2 * self.M * self.N * nb

    def library(self):
        import torch
        a = self.A.transpose(1, 2)            # batch x M x K views of column-major A
        b = self.B.transpose(1, 2)            # batch x K x N
        out = self.C.transpose(1, 2)
        return (lambda: torch.baddbmm(out, a, b, beta=0.0, alpha=1.0 / math.sqrt(self.K),
                                      out=out),
                "torch.baddbmm bf16 (NVIDIA cuBLAS strided batched), same shape/alpha")


def sub_blocks_for(n, world):
    """Sub-blocks of the overlapped N-split: the most (of 4, 2) whose column
    pieces stay multiples of 128, else 1."""
    for sb in (4, 2):
        if n % (world * sb * 128) == 0:
            return sb
    return 1


class GemmI8(Workload):
    name, dtype, unit, scaling = "gemm_i8", "int8", "TOPS", "strong"
    peak_scale = 2.0
    M, K, N = 2048, 4096, 14336
    gather = True
    # N > 1: how C is gathered.  None = the form measured fastest at this N:
    # copy-engine copies into the peers' C overlapped with the GEMM at N = 2,
    # one NCCL all-gather after the GEMM above (see overlap_for)
    overlap = None

    @classmethod
    def overlap_for(cls, world):
        return (world == 2) if cls.overlap is None else cls.overlap

    @classmethod
    def config_for(cls, world):
        if not cls.gather:
            par = f"N-split x{world}, column blocks left on their GPUs"
        elif cls.overlap_for(world) and world > 1:
            par = (f"N-split x{world} in {sub_blocks_for(cls.N, world)} sub-blocks, each "
                   f"stored into the peers' C over NVLink while the next is computed "
                   f"(zlift_part_gemm_ex_nsplit_overlap, registered C)")
        else:
            par = f"N-split x{world} + NCCL all-gather of C after the GEMM (zlift_part_gemm_ex_nsplit)"
        return {"workload": "cublasGemmEx int8->int32 M=2048 K=4096 N=14336 transa=T transb=N "
                            "alpha=1 beta=0", "m": 2048, "n": 14336, "k": 4096,
                "inputs": "A,B uniform integers in [-127,127] (seeded)",
                "l2": "inputs + output 184 MB larger than L2", "parallelism": par}

    def __init__(self, h, dev, rank, world, stream):
        import torch
        import torch.distributed as dist
        from zlift_b200 import partition
        self.h, self.world, self.rank = h, world, rank
        self.overlap = self.overlap_for(world)
        lo, hi = partition.shard_range(self.N, world, rank, align=128)
        self.n0, self.nl = lo, hi - lo
        self.A = _gen("i8", (self.M, self.K), 60, dev)                 # stored K x M (op T)
        self.B = _gen("i8", (self.nl, self.K), 70 + rank, dev)          # K x nl column block
        self.C = torch.empty(self.N, self.M, dtype=torch.int32, device=dev)   # full m x n
        # the e2e pipeline's second buffer slot
        self.slots = [(self.A, self.B, self.C),
                      tuple(torch.empty_like(t) for t in (self.A, self.B, self.C))]
        self.comm = None
        if world > 1 and self.gather:
            box = [partition.Comm.unique_id() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0)
            self.comm = partition.Comm(world, rank, box[0])
            if self.overlap:
                # the overlapped gather stores into the peers' C directly
                for _, _, C in self.slots:
                    rc = self.comm.register_peer_buffer(C, C.numel() * 4)
                    assert rc == 0, rc
        self.flops = 2.0 * self.M * self.N * self.K
        self.kernel_flops = 2.0 * self.M * self.nl * self.K
        self.kernel_bytes = float(self.M * self.K + self.K * self.nl + 4 * self.M * self.nl)
        if world > 1 and self.gather:
            self.launches_per_step = 1     # plus NCCL's own kernel
        self.hA, self.hB = self.A.cpu().pin_memory(), self.B.cpu().pin_memory()
        self.hC = [torch.empty(self.N * self.M, dtype=torch.int32).pin_memory()
                   for _ in range(2)]

    def _gemm(self, A, B, C):
        from zlift_b200 import partition
        if self.gather and self.overlap and self.world > 1:
            st = partition.gemm_ex_nsplit_overlap(
                self.h, self.comm, self.world, self.rank, sub_blocks_for(self.N, self.world), 1,
                0, self.M, self.N, self.K, 1, A, 3, self.K, B, 3, self.K, 0, C, 10, 72)
        elif self.gather:
            st = partition.gemm_ex_nsplit(self.h, self.comm, self.world, self.rank, 1, 0, self.M,
                                          self.N, self.K, 1, A, 3, self.K, B, 3, self.K, 0, C,
                                          10, 72)
        else:
            cblk = C[self.n0:self.n0 + self.nl]
            st = self.h.gemm_ex(1, 0, self.M, self.nl, self.K, 1, A, 3, self.K, B, 3, self.K, 0,
                                cblk, 10, self.M, compute=72)
        assert st == 0, st

    def step(self, i):
        self._gemm(self.A, self.B, self.C)

    def e2e_upload(self, slot):
        A, B, _ = self.slots[slot]
        A.copy_(self.hA, non_blocking=True)
        B.copy_(self.hB, non_blocking=True)

    def e2e_compute(self, slot):
        self._gemm(*self.slots[slot])

    def e2e_download(self, slot):
        C = self.slots[slot][2]
        if self.gather:
            self.hC[slot].copy_(C.view(-1), non_blocking=True)
        else:
            self.hC[slot][:self.nl * self.M].copy_(C[self.n0:self.n0 + self.nl].reshape(-1),
                                                    non_blocking=True)

    def e2e_bytes(self):
        out = 4 * self.N * self.M if self.gather else 4 * self.nl * self.M
        return self.M * self.K + self.K * self.nl, out

    def library(self):
        import torch
        a = self.A                            # M x K row-major == op(A) with A stored K x M
        b = self.B.t()                        # K x n: column block, K contiguous
        return (lambda: torch._int_mm(a, b),
                "torch._int_mm int8 (NVIDIA cuBLASLt), same M, K, N and operand layouts")

    def close(self):
        if self.comm is not None:
            import torch
            import torch.distributed as dist
            torch.cuda.synchronize()
            dist.barrier()                 # no rank still stores into another's C
            self.comm.close()


class GemmI8NoGather(GemmI8):
    name = "gemm_i8_nogather"
    gather = False


class GemmI8SerialGather(GemmI8):
    name = "gemm_i8_serialgather"
    overlap = False


class GemmI8PeerCopy(GemmI8):
    name = "gemm_i8_peercopy"
    overlap = True


class Fmha(Workload):
    name, dtype, scaling = "fmha", "bf16", "strong"
    B, H, S, D = 8, 32, 4096, 128

    @staticmethod
    def config_for(world):
        return {"workload": "flash attention forward bf16 B=8 H=32 Sq=Sk=4096 D=128 causal "
                            "scale=1/sqrt(128), bf16 O + fp32 LSE, BSHD", "batch": 8,
                "heads": 32, "seq": 4096, "head_dim": 128, "inputs": "Q,K,V ~ N(0,1) (seeded)",
                "l2": "inputs 768 MiB larger than L2",
                "parallelism": f"(batch,head)-split x{world} (zlift_part_flash_fwd)"}

    def __init__(self, h, dev, rank, world, stream):
        import torch
        from zlift_b200 import partition
        self.stream, self.world = stream, world
        lo, hi = partition.shard_range(self.B * self.H, world, rank)
        self.lo, self.hi = lo, hi
        # each rank holds the batches its (batch, head) range touches
        b0, b1 = lo // self.H, (hi + self.H - 1) // self.H
        self.b0, self.nbl = b0, max(b1 - b0, 0)
        shape = (max(self.nbl, 1), self.S, self.H, self.D)
        self.q = _gen("bf16", shape, 80, dev)
        self.k = _gen("bf16", shape, 81, dev)
        self.v = _gen("bf16", shape, 82, dev)
        self.o = torch.empty_like(self.q)
        self.lse = torch.empty(shape[0], self.H, self.S, dtype=torch.float32, device=dev)
        full = 4.0 * self.S * self.S * self.D / 2.0       # causal half, QK^T + PV
        self.flops = full * self.B * self.H
        self.kernel_flops = full * (hi - lo)
        self.kernel_bytes = (hi - lo) * (4 * 2 * self.S * self.D + 4 * self.S)
        self.hq, self.hk, self.hv = (t.cpu().pin_memory() for t in (self.q, self.k, self.v))
        self.ho = [torch.empty_like(self.o, device="cpu").pin_memory() for _ in range(2)]
        from zlift_b200 import attention
        self.blk = attention.flash_block(self.q, self.k, self.v, self.o, self.lse, causal=True)
        # the e2e pipeline's second buffer slot
        q2, k2, v2, o2, l2 = (torch.empty_like(t) for t in (self.q, self.k, self.v, self.o,
                                                            self.lse))
        self.slots = [(self.q, self.k, self.v, self.o, self.blk),
                      (q2, k2, v2, o2, attention.flash_block(q2, k2, v2, o2, l2, causal=True))]
        self._lse2 = l2

    def _run(self, blk):
        from zlift_b200 import partition
        if self.hi <= self.lo:
            return
        rc = partition.flash_pairs(blk, 1, self.lo - self.b0 * self.H,
                                   self.hi - self.b0 * self.H, self.stream)
        assert rc == 0, rc

    def step(self, i):
        self._run(self.blk)

    def e2e_upload(self, slot):
        for d, hsrc in zip(self.slots[slot][:3], (self.hq, self.hk, self.hv)):
            d.copy_(hsrc, non_blocking=True)

    def e2e_compute(self, slot):
        self._run(self.slots[slot][4])

    def e2e_download(self, slot):
        self.ho[slot].copy_(self.slots[slot][3], non_blocking=True)

    def e2e_bytes(self):
        n = self.q.numel() * 2
        return 3 * n, n

    def library(self):
        import torch
        import torch.nn.functional as F
        q, k, v = (t.transpose(1, 2) for t in (self.q, self.k, self.v))   # B H S D views

        def run():
            with torch.nn.attention.sdpa_kernel([torch.nn.attention.SDPBackend.CUDNN_ATTENTION,
                                                 torch.nn.attention.SDPBackend.FLASH_ATTENTION]):
                return F.scaled_dot_product_attention(q, k, v, is_causal=True)
        return run, "torch scaled_dot_product_attention bf16 causal (cuDNN / flash backend)"


class Sgemm(Workload):
    name, dtype = "sgemm", "f32"
    M = N = K = 1024
    peak_scale = None       # no tensor-core peak is measured for the 3-product fp32 path

    @staticmethod
    def config_for(world):
        return {"workload": "cublasSgemm_v2 fp32 M=N=K=1024 NN alpha=1 beta=0 (3-product "
                            "tf32 split, fp32 accuracy)", "m": 1024, "n": 1024, "k": 1024,
                "inputs": "A,B ~ U[-1,1) (seeded)",
                "l2": "40 rotating input sets (480 MiB)", "parallelism": f"replicas x{world}"}

    def __init__(self, h, dev, rank, world, stream):
        import torch
        self.h, self.world = h, world
        M = self.M
        g = torch.Generator(device=dev).manual_seed(90)
        self.sets = []
        for s in range(40):          # 40 x 12 MiB rotating sets > L2
            A = torch.rand(M, M, device=dev, generator=g) * 2 - 1
            B = torch.rand(M, M, device=dev, generator=g) * 2 - 1
            C = torch.zeros(M, M, device=dev)
            self.sets.append((A, B, C))
        self.flops = 2.0 * M ** 3 * world
        self.kernel_flops = 2.0 * M ** 3
        self.kernel_bytes = 3 * 4 * M * M
        self.launches_per_step = 3   # two tf32 split kernels + the GEMM
        self.hA, self.hB = self.sets[0][0].cpu().pin_memory(), self.sets[0][1].cpu().pin_memory()
        self.hC = [torch.empty(M, M).pin_memory() for _ in range(2)]

    def step(self, i):
        A, B, C = self.sets[i % len(self.sets)]
        st = self.h.sgemm(0, 0, self.M, self.N, self.K, 1.0, A, self.M, B, self.K, 0.0, C, self.M)
        assert st == 0, st

    def e2e_upload(self, slot):
        A, B, _ = self.sets[slot]
        A.copy_(self.hA, non_blocking=True)
        B.copy_(self.hB, non_blocking=True)

    def e2e_compute(self, slot):
        self.step(slot)

    def e2e_download(self, slot):
        self.hC[slot].copy_(self.sets[slot][2], non_blocking=True)

    def e2e_bytes(self):
        return 8 * self.M * self.M, 4 * self.M * self.M

    def library(self):
        import torch
        A, B, C = self.sets[0]

        def run():
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = False
            try:
                return torch.mm(A, B, out=C)
            finally:
                torch.backends.cuda.matmul.allow_tf32 = prev
        return run, "torch.mm fp32, TF32 off (NVIDIA cuBLAS)"


WORKLOADS = {w.name: w for w in (GemmF16, GemmBF16Batched, GemmI8, GemmI8NoGather,
                                 GemmI8SerialGather, GemmI8PeerCopy, Fmha, Sgemm)}


# --------------------------------------------------------------------------
# CPU baseline (reference zblas.c build, or the oracle restatement)
# --------------------------------------------------------------------------

def cpu_reference(workload: str, steps: int, warmup: int, budget_s: float):
    """Times the reference CPU path on a bounded sample.  Returns
    (value, unit, cores, kind, sample description)."""
    from oracle import oracle
    cores = _CORES
    rng = np.random.default_rng(0)
    unit = "TOPS" if workload.startswith("gemm_i8") else "TFLOP/s"
    if workload == "fmha":
        B, H, S, D = 8, 32, 4096, 128
        from zlift_b200 import inputs
        qb = inputs.to_bf16_bits(rng.standard_normal((1, S, 1, D)).astype(np.float32)).reshape(1, S, 1, D)
        kb = inputs.to_bf16_bits(rng.standard_normal((1, S, 1, D)).astype(np.float32)).reshape(1, S, 1, D)
        vb = inputs.to_bf16_bits(rng.standard_normal((1, S, 1, D)).astype(np.float32)).reshape(1, S, 1, D)
        # query rows spread over the sequence (causal cost grows with the row index)
        nrows = 256
        rows = np.linspace(0, S - 1, nrows).astype(np.int32)
        z = np.zeros(nrows, np.int32)
        call = lambda: oracle.attention_rows(qb, kb, vb, True, 1 / math.sqrt(D), 1, z, z, rows)
        flops = float(np.sum(4.0 * (rows + 1) * D))       # row i sees i+1 keys
        kind = "port"
        sample = (f"{nrows} query rows of one (batch, head), spread over S=4096, through the "
                  f"oracle's C restatement (the reference has no CPU attention path)")
    else:
        oracle.build(ref=True)
        kind = "reference" if oracle.ref_available() else "port"
        if workload == "gemm_f16":
            M = N = K = 4096
            A = (rng.standard_normal(M * K) / 64).astype(np.float16).view(np.uint16)
            B = (rng.standard_normal(N * K) / 64).astype(np.float16).view(np.uint16)
            C = rng.standard_normal(M * N).astype(np.float16).view(np.uint16)
            fn = oracle.ref_gemm_ex if kind == "reference" else oracle.gemm_ex
            call = lambda: fn(0, 1, M, N, K, 1.0, A, 2, M, B, 2, N, 0.5, C, 2, M)
            flops = 2.0 * M * N * K
            sample = "one full 4096^3 fp16 cublasGemmEx per step (host widen + cblas_sgemm + narrow)"
        elif workload == "gemm_bf16_batched":
            M = N = K = 512
            nb = 16
            A = inputs_bf16(rng, M * K * nb)
            B = inputs_bf16(rng, M * K * nb)
            C = np.zeros(M * N * nb, np.uint16)
            fn = (oracle.ref_gemm_strided_batched_ex if kind == "reference"
                  else oracle.gemm_strided_batched_ex)
            call = lambda: fn(0, 0, M, N, K, 1 / math.sqrt(K), A, 14, M, M * K, B, 14, K, K * N,
                              0.0, C, 14, M, M * N, nb)
            flops = 2.0 * M * N * K * nb
            sample = "16 of the 256 batched 512^3 bf16 GEMMs per step (reference host loop)"
        elif workload.startswith("gemm_i8"):
            M, K, N = 2048, 4096, 1024
            A = rng.integers(-127, 128, M * K).astype(np.int8)
            B = rng.integers(-127, 128, N * K).astype(np.int8)
            C = np.zeros(M * N, np.int32)
            call = lambda: oracle.gemm_ex(1, 0, M, N, K, 1, A, 3, K, B, 3, K, 0, C, 10, M, 72)
            kind = "port"   # the reference answers int8 with NOT_SUPPORTED
            flops = 2.0 * M * N * K
            sample = ("N=1024 column block of the 2048x4096x14336 int8 GEMM per step (oracle "
                      "restatement, vectorised int32 dot products; the reference has no int8 "
                      "GEMM)")
        else:
            M = N = K = 1024
            A = rng.uniform(-1, 1, M * K).astype(np.float32)
            B = rng.uniform(-1, 1, M * K).astype(np.float32)
            C = np.zeros(M * N, np.float32)
            if kind == "reference":
                call = lambda: oracle.ref_sgemm(0, 0, M, N, K, 1.0, A, M, B, K, 0.0, C, M)
            else:
                call = lambda: oracle.gemm_ex(0, 0, M, N, K, 1.0, A, 0, M, B, 0, K, 0.0, C, 0, M)
            flops = 2.0 * M ** 3
            sample = "one full 1024^3 cublasSgemm_v2 per step"
    t_start = time.perf_counter()
    for _ in range(max(warmup, 1)):
        call()
        if time.perf_counter() - t_start > budget_s / 3:
            break
    times = []
    t_start = time.perf_counter()
    for _ in range(max(steps, 1)):
        t0 = time.perf_counter()
        call()
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > budget_s:
            break
    dt = statistics.median(times)
    return flops / dt / 1e12, unit, cores, kind, sample + f" ({len(times)} timed, median)"


def inputs_bf16(rng, n):
    from zlift_b200 import inputs
    return inputs.to_bf16_bits(rng.standard_normal(n).astype(np.float32))


# --------------------------------------------------------------------------

def time_library(w, warmup: int, steps: int, reps: int):
    """Same-box vendor-library figure for the workload (diagnostic only),
    timed like our own arm: `reps` regions of `steps` back-to-back calls on
    one stream, median region."""
    import torch
    try:
        fn, what = w.library()
    except Exception as e:               # no library form for this workload
        return {"unavailable": str(e)[:200]}
    try:
        for _ in range(max(warmup, 2)):
            fn()
        torch.cuda.synchronize()
        ts = []
        for _ in range(reps):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(steps):
                fn()
            e1.record()
            e1.synchronize()
            ts.append(e0.elapsed_time(e1) / steps)
        ms = statistics.median(ts)
        return {"value": w.kernel_flops / (ms * 1e-3) / 1e12, "unit": w.unit, "ms": ms,
                "what": what, "timing": f"median of {reps} regions of {steps} back-to-back "
                                        f"calls"}
    except Exception as e:
        torch.cuda.synchronize()
        return {"unavailable": f"{what}: {str(e)[:200]}"}


def run_workload(W, h, dev, rank, world, local, stream, steps, warmup, clk, pk, src, cpu,
                 library):
    import torch
    import torch.distributed as dist
    from zlift_b200 import blas

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        t = torch.tensor([x], dtype=torch.float64, device=dev)
        if world > 1:
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    with torch.cuda.stream(stream):
        w = W(h, dev, rank, world, stream)
    torch.cuda.synchronize()
    with torch.cuda.stream(stream):
        w.step(0)                     # first call: module loading, tensor maps
        torch.cuda.synchronize()
        t0 = time.perf_counter()
        for i in range(1, warmup):
            w.step(i)
    torch.cuda.synchronize()
    warm_s = (time.perf_counter() - t0) / max(warmup - 1, 1)
    # repeats of the K-step region: the clock record should cover at least
    # ~0.3 s under load; the same count on every rank
    reps = int(min(100, max(3, math.ceil(0.3 / max(warm_s * steps, 1e-6)))))
    reps = int(max_over_ranks(reps))

    launches0 = blas.launch_count()
    rep_ms = []
    windows = []
    for r in range(reps):
        t_start = torch.cuda.Event(enable_timing=True)
        t_end = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        with torch.cuda.stream(stream):
            t_start.record(stream)
            for i in range(steps):
                w.step(i)
            t_end.record(stream)
        torch.cuda.synchronize()
        windows.append((w0, time.perf_counter()))
        barrier()
        rep_ms.append(max_over_ranks(t_start.elapsed_time(t_end)))
    launches = (blas.launch_count() - launches0) // reps
    assert blas.device_error() == 0
    ms_total = statistics.median(rep_ms)
    ms_per_step = ms_total / steps
    value = w.flops / (ms_per_step * 1e-3) / 1e12

    # Per-call durations, in a separate pass: an event recorded between two
    # calls makes the stream finish the first before it starts the second,
    # which exposes the launch latency the back-to-back region above hides
    # (up to ~15 us per call for the batched GEMM), so the timed region
    # carries no per-step events.
    per_step = []
    for r in range(min(reps, 5)):
        starts = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        ends = [torch.cuda.Event(enable_timing=True) for _ in range(steps)]
        barrier()
        torch.cuda.synchronize()
        with torch.cuda.stream(stream):
            for i in range(steps):
                starts[i].record(stream)
                w.step(i)
                ends[i].record(stream)
        torch.cuda.synchronize()
        barrier()
        per_step.extend(a.elapsed_time(b) for a, b in zip(starts, ends))
    per_call_ms = statistics.mean(per_step)
    if world == 1:
        # the dominant kernel's average duration is at most the back-to-back
        # region's time per step (which also holds the gaps between launches
        # and, for the fp32 GEMM, its two tf32 split kernels)
        kernel_ms = ms_per_step
        kernel_how = ("timed region (CUDA events at its ends) / steps"
                      + ("" if w.launches_per_step == 1 else
                         f" ({w.launches_per_step} launches per step, all counted)"))
    else:
        kernel_ms = per_call_ms
        kernel_how = "per-step CUDA events around each call" + (
            " (GEMM + NCCL all-gather)"
            if (w.name.startswith("gemm_i8") and w.gather and world > 1) else "")

    # ---- e2e through the same C ABI with host buffers ----
    # Every step uploads its inputs from pinned host memory, runs, and
    # downloads its result.  Pipelined (the reported figure): two device
    # buffer slots, uploads on one copy stream and downloads on another, so
    # step i+1's upload runs while step i computes and downloads (PCIe is
    # full duplex); a slot is re-uploaded only after its previous result has
    # been downloaded.  Serial (reported beside it): one slot, each step's
    # upload, kernel and download in order on one stream.
    e2e_steps = max(4, min(20, steps))
    s_in = torch.cuda.Stream(device=dev)
    s_out = torch.cuda.Stream(device=dev)

    def e2e_pipelined(n):
        up = [torch.cuda.Event() for _ in range(2)]
        done = [torch.cuda.Event() for _ in range(2)]
        down = [torch.cuda.Event() for _ in range(2)]
        begin = torch.cuda.Event()
        begin.record(stream)
        s_in.wait_event(begin)
        s_out.wait_event(begin)
        for i in range(n):
            slot = i % 2
            if i >= 2:
                s_in.wait_event(down[slot])
            with torch.cuda.stream(s_in):
                w.e2e_upload(slot)
            up[slot].record(s_in)
            stream.wait_event(up[slot])
            with torch.cuda.stream(stream):
                w.e2e_compute(slot)
            done[slot].record(stream)
            s_out.wait_event(done[slot])
            with torch.cuda.stream(s_out):
                w.e2e_download(slot)
            down[slot].record(s_out)
        for slot in range(min(n, 2)):
            stream.wait_event(down[slot])

    def e2e_serial(n):
        with torch.cuda.stream(stream):
            for _ in range(n):
                w.e2e_upload(0)
                w.e2e_compute(0)
                w.e2e_download(0)

    def e2e_time(fn):
        fn(2)                                   # warm both slots and streams
        torch.cuda.synchronize()
        e0 = torch.cuda.Event(enable_timing=True)
        e1 = torch.cuda.Event(enable_timing=True)
        barrier()
        torch.cuda.synchronize()
        e0.record(stream)
        fn(e2e_steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = max_over_ranks(e0.elapsed_time(e1) / e2e_steps)
        barrier()
        return ms

    e2e_ms = e2e_time(e2e_pipelined)
    e2e_serial_ms = e2e_time(e2e_serial)
    bi, bo = w.e2e_bytes()

    rec = None
    lib = None
    if rank == 0 and library and world == 1:
        with torch.cuda.stream(stream):
            lib = time_library(w, warmup, steps, reps)
    if rank == 0:
        clocks = clk.summary(windows)
        # the sustained (power-capped) GEMM figure is the denominator only
        # when the region actually ran below full clock; a region at full
        # clock is compared with the burst figure
        slow = (clocks["sm_mhz"] is not None and clocks["sm_max_mhz"]
                and clocks["sm_mhz"] < 0.95 * clocks["sm_max_mhz"])
        sustained = bool(slow) and "bf16_tflops_sustained" in pk
        if w.bound == "hbm":
            achieved = w.kernel_bytes / (kernel_ms * 1e-3) / 1e9
            peak, unit_r, peak_key = pk["hbm_gbs"], "GB/s", "hbm_gbs"
        else:
            achieved = w.kernel_flops / (kernel_ms * 1e-3) / 1e12
            peak_key = "bf16_tflops_sustained" if sustained else "bf16_tflops"
            # 3-product tf32 fp32 GEMM: tf32 runs at half the bf16 rate and
            # every output term takes three products
            scale = w.peak_scale if w.peak_scale is not None else 1.0 / 6.0
            peak, unit_r = pk[peak_key] * scale, "TFLOP/s"
            if w.unit == "TOPS":
                unit_r = "TOPS"
        rec = {
            "value": value, "unit": w.unit, "ms_per_step": ms_per_step,
            "repeats": reps, "ms_per_step_repeats": [min(rep_ms) / steps, ms_per_step,
                                                     max(rep_ms) / steps],
            "scaling": w.scaling, "dtype": w.dtype, "config": w.config(),
            "roofline": {"bound": w.bound, "achieved": achieved, "peak": peak,
                         "unit": unit_r, "frac": achieved / peak,
                         "peak_source": f"{src} {peak_key}"
                                        + (f" x{w.peak_scale:g} (int8 dense rate = 2 x bf16)"
                                           if (w.peak_scale or 1) != 1 else "")
                                        + ("" if w.peak_scale is not None else
                                           " / 6 (tf32 = 1/2 of the bf16 rate, 3 products "
                                           "per output term; frac per useful fp32 FLOP)"),
                         "traffic": traffic_from_profile(w.name) if world == 1 else None,
                         "kernel_ms": kernel_ms,
                         "kernel": kernel_how,
                         "per_call_events_ms": per_call_ms},
            "e2e": {"value": w.flops / (e2e_ms * 1e-3) / 1e12, "unit": w.unit,
                    "h2d_bytes_per_step": bi, "d2h_bytes_per_step": bo, "ms_per_step": e2e_ms,
                    "steps": e2e_steps,
                    "timing": "pipelined over 2 buffer slots: upload (copy stream) -> kernel "
                              "-> download (second copy stream); every step copies its own "
                              "inputs and result",
                    "serial_ms_per_step": e2e_serial_ms,
                    "serial_value": w.flops / (e2e_serial_ms * 1e-3) / 1e12},
            "gpu_launches": int(launches),
            "clocks": clocks,
        }
        if lib is not None:
            rec["library_same_box"] = lib
        if cpu and world == 1:
            v, unit, cores, kind, sample = cpu_reference(w.name, 5, 1, budget_s=12.0)
            rec["cpu_baseline"] = {"value": v, "unit": unit, "cores": cores, "kind": kind,
                                   "sample": sample}
    torch.cuda.synchronize()
    w.close()
    del w
    torch.cuda.empty_cache()
    return rec, windows


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="all", choices=["all"] + sorted(WORKLOADS))
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-library", action="store_true")
    a = ap.parse_args(argv)
    warmup = max(a.warmup, 3)
    steps = max(a.steps, 1)

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    names = ORDER if a.workload == "all" else [a.workload]
    nw = max(world, a.gpus)
    if a.workload == "all" and nw > 1:
        # the int8 gather form gemm_i8 does not use, and no gather at all
        names = names + ["gemm_i8_serialgather" if nw == 2 else "gemm_i8_peercopy",
                         "gemm_i8_nogather"]
    head = HEADLINE if HEADLINE in names else names[0]

    if a.impl == "reference":
        if rank != 0:
            return 0
        recs = {}
        for n in names:
            W = WORKLOADS[n]
            v, unit, cores, kind, sample = cpu_reference(n, steps, warmup, budget_s=15.0)
            recs[n] = {"value": v, "unit": unit, "scaling": W.scaling, "dtype": W.dtype,
                       "config": W.config_for(a.gpus),
                       "cpu_baseline": {"value": v, "unit": unit, "cores": cores, "kind": kind,
                                        "sample": sample},
                       "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0,
                               "d2h_bytes_per_step": 0}}
        hr = recs[head]
        line = {"metric": METRIC, "value": hr["value"], "unit": hr["unit"], "n_gpus": a.gpus,
                "steps": steps, "warmup": warmup, "ms_per_step": None,
                "higher_is_better": True, "scaling": hr["scaling"], "vs_baseline": None,
                "dtype": hr["dtype"], "data": "synthetic (seeded, benchmark shapes)",
                "impl": "reference", "config": hr["config"],
                "cpu_baseline": hr["cpu_baseline"], "e2e": hr["e2e"],
                "configs": recs}
        print(json.dumps(line), flush=True)
        return 0

    import torch
    import torch.distributed as dist
    from zlift_b200 import blas

    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    stream = torch.cuda.Stream(device=dev)
    h = blas.Handle(stream)
    pk, src = peaks()
    clk = ClockSampler(local)
    clk.start()
    recs, all_windows = {}, []
    try:
        for n in names:
            rec, windows = run_workload(WORKLOADS[n], h, dev, rank, world, local, stream, steps,
                                        warmup, clk, pk, src, cpu=not a.no_cpu_baseline,
                                        library=not a.no_library)
            all_windows.extend(windows)
            if rank == 0:
                recs[n] = rec
    finally:
        clk.stop()
    if rank == 0:
        hr = recs[head]
        line = {"metric": METRIC, "value": hr["value"], "unit": hr["unit"], "n_gpus": world,
                "steps": steps, "warmup": warmup, "ms_per_step": hr["ms_per_step"],
                "higher_is_better": True, "scaling": hr["scaling"], "vs_baseline": None,
                "dtype": hr["dtype"],
                "data": "synthetic (seeded torch generator, benchmark shapes)",
                "config": hr["config"], "roofline": hr["roofline"], "e2e": hr["e2e"],
                "gpu_launches": hr["gpu_launches"],
                # the clock record of every timed region of the run (all configurations)
                "clocks": clk.summary(all_windows),
                "repeats": hr["repeats"]}
        if "cpu_baseline" in hr:
            line["cpu_baseline"] = hr["cpu_baseline"]
        if "library_same_box" in hr:
            line["library_same_box"] = hr["library_same_box"]
        line["configs"] = recs
        print(json.dumps(line), flush=True)
    torch.cuda.synchronize()
    h.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
