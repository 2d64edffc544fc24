"""K-split of the GEMM kernel's last wave, on the GPU.

When the last wave of output tiles would leave more than half of the
persistent CTAs idle, the tensor-core kernel splits each of its tiles along
K into 2-4 parts run by different CTAs, and the part that finishes last sums
the parts' fp32 (or int32) partials in part order before the epilogue.  The
shapes below are chosen so that a split happens (the tile count modulo the
148 CTAs, or 74 CTA pairs, is at most half of them), and each result is
compared with the oracle on the same seeded inputs: bit-exact for int8,
normwise <= 1e-2 for 16-bit inputs and <= 1e-5 for fp32.  The split is
switched on with ZBLAS_SPLIT_K=1 (module fixture) and off with
ZBLAS_SPLIT_K=0 for the split-versus-whole comparisons.
"""
import os

import numpy as np
import pytest

from tests.helpers import CUDA_T, as_float, from_dev, normwise, to_dev
from tests.test_gemm_gpu import run_gemm

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def handle(cuda):
    from zlift_b200 import Handle
    old = os.environ.get("ZBLAS_SPLIT_K")
    os.environ["ZBLAS_SPLIT_K"] = "1"
    try:
        with Handle() as h:
            yield h
    finally:
        if old is None:
            os.environ.pop("ZBLAS_SPLIT_K", None)
        else:
            os.environ["ZBLAS_SPLIT_K"] = old


class _Env:
    """Sets environment variables for the duration of a with-block (the
    library reads its switches at each call)."""

    def __init__(self, **kv):
        self.kv = kv
        self.old = {}

    def __enter__(self):
        for k, v in self.kv.items():
            self.old[k] = os.environ.get(k)
            os.environ[k] = v

    def __exit__(self, *exc):
        for k, v in self.old.items():
            if v is None:
                os.environ.pop(k, None)
            else:
                os.environ[k] = v


# 16 tiles of 128 x 128 on 148 CTAs: 4 parts of 32 K blocks each
def test_split_int8_bit_exact(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "i8", "i32", 1, 0, 256, 1024, 8192, 3, -2, dist="int8")


@pytest.mark.parametrize("ta,tb", [(0, 1), (1, 0), (0, 0)])
def test_split_f16_beta(handle, oracle_lib, ta, tb):
    run_gemm(handle, oracle_lib, "f16", "f16", ta, tb, 512, 512, 8192, 1.0, 0.5, seed=11,
             scale=0.125)


def test_split_ragged_k_and_edges(handle, oracle_lib):
    """K not a multiple of the 64-element K block, M and N not multiples of
    the tile: the parts get unequal K ranges and the edge tiles are clipped."""
    run_gemm(handle, oracle_lib, "bf16", "bf16", 0, 0, 300, 420, 5000, 0.5, 0.25, seed=12,
             scale=0.125)


def test_split_f32_out(handle, oracle_lib):
    run_gemm(handle, oracle_lib, "bf16", "f32", 1, 1, 384, 256, 4096, 1.0, 1.0, seed=13)


def test_split_sgemm(handle, oracle_lib):
    """fp32 (3xTF32 kernel, 4 parts) at K = 8192, against an fp64 product of
    the same inputs and against the oracle's fp32 result: the tensor core's
    fp32 accumulation loses precision at every step, so the kernel starts a
    fresh accumulator every 128 of K and adds the chunks in fp32, round to
    nearest; without that the error reached 5e-5 at this K."""
    from zlift_b200 import inputs
    m, n, k = 256, 256, 8192
    A = inputs.make("f32", "uniform", 14, m * k)
    B = inputs.make("f32", "uniform", 15, k * n)
    exact = (A.astype(np.float64).reshape(k, m).T @ B.astype(np.float64).reshape(n, k).T)
    exact = exact.T.reshape(-1)
    cref = np.zeros(m * n, np.float32)
    assert oracle_lib.gemm_ex(0, 0, m, n, k, 1.0, A, 0, m, B, 0, k, 0.0, cref, 0, m) == 0
    dA, dB = to_dev(A, "f32"), to_dev(B, "f32")
    dC = to_dev(np.zeros(m * n, np.float32), "f32")
    assert handle.sgemm(0, 0, m, n, k, 1.0, dA, m, dB, k, 0.0, dC, m) == 0
    got = from_dev(dC, "f32").astype(np.float64)
    err_gpu = normwise(got, exact)
    err_oracle = normwise(cref.astype(np.float64), exact)
    assert err_gpu <= 2e-6, (err_gpu, err_oracle)
    assert normwise(got, cref.astype(np.float64)) <= 1e-5


@pytest.mark.parametrize("kind", ["f16", "i8"])
def test_split_pair_tiles(handle, oracle_lib, kind):
    """CTA-pair kernel forced: 4 x 8 pair tiles of 256 x 256 on 74 pairs, 2
    parts each; each CTA of a pair keeps its own partials and counter."""
    with _Env(ZBLAS_GEMM_CFG="p256"):
        if kind == "i8":
            run_gemm(handle, oracle_lib, "i8", "i32", 1, 0, 1024, 2048, 4096, 1, 0, dist="int8")
        else:
            run_gemm(handle, oracle_lib, "f16", "f16", 0, 1, 1024, 2048, 4096, 1.0, 0.5,
                     seed=15, scale=0.125)


def test_split_strided_batched(handle, oracle_lib):
    from zlift_b200 import inputs
    m, n, k, batch = 256, 256, 4096, 3
    A = inputs.make("bf16", "normal", 31, m * k * batch, 0.125)
    B = inputs.make("bf16", "normal", 32, k * n * batch, 0.125)
    C0 = inputs.make("bf16", "normal", 33, m * n * batch)
    cref = C0.copy()
    assert oracle_lib.gemm_strided_batched_ex(0, 0, m, n, k, 1.0, A, 14, m, m * k, B, 14, k,
                                              k * n, 0.5, cref, 14, m, m * n, batch) == 0
    dA, dB, dC = to_dev(A, "bf16"), to_dev(B, "bf16"), to_dev(C0, "bf16")
    assert handle.gemm_strided_batched_ex(0, 0, m, n, k, 1.0, dA, 14, m, m * k, dB, 14, k,
                                          k * n, 0.5, dC, 14, m, m * n, batch) == 0
    got = as_float(from_dev(dC, "bf16"), "bf16")
    assert normwise(got, as_float(cref, "bf16")) <= 1e-2


def test_split_matches_whole_tiles(handle, cuda):
    """The bench shape (4096^3 fp16 NT, 256 pair tiles on 74 pairs, 34 tiles
    in the last wave, 2 parts each): split and unsplit results differ only
    by fp32 summation order, and each is bitwise repeatable."""
    import torch
    from zlift_b200 import inputs
    m = n = k = 4096
    A = to_dev(inputs.make("f16", "normal", 41, m * k, 1 / 64), "f16")
    B = to_dev(inputs.make("f16", "normal", 42, k * n, 1 / 64), "f16")
    C0 = to_dev(inputs.make("f16", "normal", 43, m * n), "f16")

    def run():
        C = C0.clone()
        assert handle.gemm_ex(0, 1, m, n, k, 1.0, A, 2, m, B, 2, n, 0.5, C, 2, m) == 0
        return C

    split = [run() for _ in range(2)]
    with _Env(ZBLAS_SPLIT_K="0"):
        whole = run()
    torch.cuda.synchronize()
    assert torch.equal(split[0], split[1])
    d = (split[0].float() - whole.float()).abs().max().item()
    assert d <= 2e-3 * whole.float().abs().max().item()
    from zlift_b200 import blas
    assert blas.device_error() == 0


def test_split_cuda_graph_replays(handle, oracle_lib, cuda):
    """A split GEMM captured in a CUDA graph (same epoch at every replay):
    the last part resets its counter, so every replay writes C."""
    import torch
    from zlift_b200 import inputs
    m, n, k = 512, 512, 8192
    A = inputs.make("f16", "normal", 51, m * k, 0.125)
    B = inputs.make("f16", "normal", 52, k * n, 0.125)
    cref = np.zeros(m * n, np.uint16)
    assert oracle_lib.gemm_ex(0, 0, m, n, k, 1.0, A, 2, m, B, 2, k, 0.0, cref, 2, m) == 0
    dA, dB = to_dev(A, "f16"), to_dev(B, "f16")
    dC = torch.zeros(m * n, dtype=torch.float16, device=cuda)
    assert handle.gemm_ex(0, 0, m, n, k, 1.0, dA, 2, m, dB, 2, k, 0.0, dC, 2, m) == 0
    first = dC.clone()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        handle.set_stream(s)
        # one eager call on the capture stream first: a stream's K-split
        # workspace is allocated on its first GEMM, never inside a capture
        assert handle.gemm_ex(0, 0, m, n, k, 1.0, dA, 2, m, dB, 2, k, 0.0, dC, 2, m) == 0
        s.synchronize()
        with torch.cuda.graph(g, stream=s):
            assert handle.gemm_ex(0, 0, m, n, k, 1.0, dA, 2, m, dB, 2, k, 0.0, dC, 2, m) == 0
    handle.set_stream(torch.cuda.current_stream())
    for _ in range(3):
        dC.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(dC, first)
    del g
    got = as_float(from_dev(dC, "f16"), "f16")
    assert normwise(got, as_float(cref, "f16")) <= 1e-2


def test_split_lt_bias_gelu(handle, built_lib, oracle_lib, cuda):
    """cublasLtMatmul with GELU_BIAS on a split shape: the last part applies
    the fused epilogue to the summed partials."""
    from tests.test_lt import test_lt_matmul_epilogues
    test_lt_matmul_epilogues(built_lib, oracle_lib, cuda, "bf16", 0, 1, 256, 512, 8192, 36,
                             1.0, 0.5, False, 1)
