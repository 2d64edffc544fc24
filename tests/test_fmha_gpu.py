"""Fused attention forward parity on the GPU, through the C ABI
(zlift_flash_fwd / zlift_fmha_fwd in libcublas.so.13), against the oracle's
restatement of the reference attention math (fmha_f32 / fmha_run).

Tolerances: O normwise (max|x - ref| / max|ref|) <= 1e-2 for 16-bit inputs
and <= 2e-5 for fp32 inputs (the reference's fmha_f32 path, elem 2); LSE
absolute <= 1e-3 (LSE is about log(S) ~ 8, so this is ~1e-4 relative;
<= 1e-5 for fp32).  The reference never produces LSE, so the LSE checks pin
it against the restatement only.
"""
import math

import numpy as np
import pytest

from tests.helpers import as_float, from_dev, normwise, to_dev

pytestmark = pytest.mark.gpu

O_TOL = 1e-2
LSE_TOL = 1e-3


def _qkv(kind, B, Sq, Sk, H, Hk, D, seed):
    from zlift_b200 import inputs
    q = inputs.make(kind, "normal", seed, B * Sq * H * D).reshape(B, Sq, H, D)
    k = inputs.make(kind, "normal", seed + 1, B * Sk * Hk * D).reshape(B, Sk, Hk, D)
    v = inputs.make(kind, "normal", seed + 2, B * Sk * Hk * D).reshape(B, Sk, Hk, D)
    return q, k, v


def _dev4(a, kind):
    return to_dev(a, kind).view(*a.shape)


def run_flash(oracle, kind, B, Sq, Sk, H, Hk, D, causal, seed=1, api="flash", bias=False):
    import torch
    import zlift_b200
    from zlift_b200 import blas, inputs
    q, k, v = _qkv(kind, B, Sq, Sk, H, Hk, D, seed)
    scale = 1.0 / math.sqrt(D)
    elem = {"bf16": 1, "f16": 0, "f32": 2}[kind]
    bh = None
    if bias:
        bh = inputs.make(kind, "normal", seed + 9, B * H * Sq * Sk).reshape(B, H, Sq, Sk)
    o_ref, lse_ref = oracle.attention(q, k, v, causal, scale, elem, kv_ratio=H // Hk, bias=bh)
    dq, dk, dv = _dev4(q, kind), _dev4(k, kind), _dev4(v, kind)
    do = torch.full_like(dq, float("nan"))
    dl = torch.full((B, H, Sq), float("nan"), dtype=torch.float32, device=dq.device)
    if api == "flash":
        rc = zlift_b200.flash_forward(dq, dk, dv, do, dl, causal=causal, scale=scale)
    else:
        db = _dev4(bh, kind) if bias else None
        rc = zlift_b200.fmha_forward(dq, dk, dv, do, dl, mask_type=2 if causal else 0,
                                     scale=scale, bias=db)
    assert rc == 0, f"entry returned {rc}"
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    o = from_dev(do.reshape(-1), kind).reshape(q.shape)
    got, want = as_float(o, kind), as_float(o_ref, kind)
    assert np.all(np.isfinite(got))
    err = normwise(got, want)
    o_tol, lse_tol = (2e-5, 1e-5) if kind == "f32" else (O_TOL, LSE_TOL)
    assert err <= o_tol, f"O normwise error {err:.3e}"
    lse = dl.cpu().numpy()
    fin = np.isfinite(lse_ref)
    np.testing.assert_array_equal(np.isfinite(lse), fin)
    if fin.any():
        assert np.max(np.abs(lse[fin] - lse_ref[fin])) <= lse_tol
    return err


@pytest.mark.parametrize("kind", ["bf16", "f16"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,S,H,D", [(1, 128, 1, 128), (1, 256, 2, 128), (2, 384, 2, 128),
                                     (1, 512, 2, 64), (1, 300, 3, 128)])
def test_flash_square(oracle_lib, cuda, kind, causal, B, S, H, D):
    run_flash(oracle_lib, kind, B, S, S, H, H, D, causal, seed=S + H)


@pytest.mark.parametrize("Sq,Sk", [(128, 384), (200, 72), (384, 128), (1, 257)])
def test_flash_causal_bottom_right(oracle_lib, cuda, Sq, Sk):
    """Sq != Sk: the causal diagonal is aligned bottom-right (diag = Sk - Sq);
    rows that see no key at all give O = 0 and LSE = -inf."""
    run_flash(oracle_lib, "bf16", 1, Sq, Sk, 2, 2, 128, True, seed=Sq)


def test_flash_gqa(oracle_lib, cuda):
    run_flash(oracle_lib, "bf16", 2, 256, 256, 8, 2, 128, True, seed=7)


@pytest.mark.parametrize("causal", [False, True])
def test_fmha_xformers_block(oracle_lib, cuda, causal):
    run_flash(oracle_lib, "bf16", 2, 256, 256, 2, 2, 128, causal, seed=3, api="fmha")


def test_declines_are_reported(cuda):
    """Unsupported requests return 1 (declined) and leave O untouched."""
    import torch
    import zlift_b200
    q = torch.zeros(1, 128, 1, 96, dtype=torch.bfloat16, device=cuda)   # head_dim 96
    o = torch.full_like(q, 3.0)
    assert zlift_b200.flash_forward(q, q, q, o, None, causal=True) == 1
    torch.cuda.synchronize()
    assert torch.all(o == 3.0)


def test_flash_full_size_sampled(oracle_lib, cuda):
    """The benchmark configuration (B=8, H=32, S=4096, D=128, causal, bf16):
    full output on the GPU, checked on 96 sampled query rows, including the
    first and last row of the sequence and of several key tiles."""
    import torch
    import zlift_b200
    B, S, H, D = 8, 4096, 32, 128
    g = torch.Generator(device=cuda).manual_seed(1234)
    q = torch.randn(B, S, H, D, generator=g, device=cuda).to(torch.bfloat16)
    k = torch.randn(B, S, H, D, generator=g, device=cuda).to(torch.bfloat16)
    v = torch.randn(B, S, H, D, generator=g, device=cuda).to(torch.bfloat16)
    o = torch.empty_like(q)
    lse = torch.empty(B, H, S, dtype=torch.float32, device=cuda)
    scale = 1.0 / math.sqrt(D)
    assert zlift_b200.flash_forward(q, k, v, o, lse, causal=True, scale=scale) == 0
    torch.cuda.synchronize()
    rng = np.random.default_rng(5)
    bs = rng.integers(0, B, 96)
    hs = rng.integers(0, H, 96)
    is_ = rng.integers(0, S, 96)
    is_[:6] = [0, 1, 127, 128, 4095, 2047]
    qh = from_dev(q.reshape(-1), "bf16").reshape(B, S, H, D)
    kh = from_dev(k.reshape(-1), "bf16").reshape(B, S, H, D)
    vh = from_dev(v.reshape(-1), "bf16").reshape(B, S, H, D)
    o_ref, l_ref = oracle_lib.attention_rows(qh, kh, vh, True, scale, 1, bs, hs, is_)
    oh = from_dev(o.reshape(-1), "bf16").reshape(B, S, H, D)
    got = as_float(oh[bs, is_, hs, :], "bf16")
    assert normwise(got, o_ref) <= O_TOL
    lg = lse.cpu().numpy()[bs, hs, is_]
    assert np.max(np.abs(lg - l_ref)) <= LSE_TOL


@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("B,Sq,Sk,H,Hk,D", [(1, 128, 128, 1, 1, 128), (2, 200, 200, 2, 2, 64),
                                            (1, 96, 300, 4, 2, 128), (1, 300, 130, 2, 1, 40),
                                            (1, 64, 64, 1, 1, 256)])
def test_flash_fp32(oracle_lib, cuda, causal, B, Sq, Sk, H, Hk, D):
    """fp32 inputs (elem 2, the reference's fmha_f32 path, zblas_gpu.cpp:793-844
    and :1367-1372): GQA, bottom-right causal, odd head dims."""
    run_flash(oracle_lib, "f32", B, Sq, Sk, H, Hk, D, causal, seed=Sq + D)


@pytest.mark.parametrize("kind", ["bf16", "f16", "f32"])
@pytest.mark.parametrize("causal", [False, True])
@pytest.mark.parametrize("Sq,Sk", [(256, 256), (200, 330)])
def test_fmha_bias(oracle_lib, cuda, kind, causal, Sq, Sk):
    """xformers block with attn_bias (zblas_gpu.cpp:963-966): the bias, of the
    input type, is added to the scaled scores before the mask."""
    run_flash(oracle_lib, kind, 2, Sq, Sk, 2, 2, 128 if kind != "f32" else 64, causal,
              seed=Sq + Sk, api="fmha", bias=True)


def test_fmha_bias_strided(oracle_lib, cuda):
    """A bias with padded rows (row stride > Sk) and heads broadcast over the
    batch: strides are honoured, rows need not be 16-byte aligned."""
    import torch
    import zlift_b200
    from zlift_b200 import blas, inputs
    B, S, H, D = 2, 256, 2, 128
    q, k, v = _qkv("bf16", B, S, S, H, H, D, 77)
    full = inputs.make("bf16", "normal", 78, H * S * (S + 3)).reshape(1, H, S, S + 3)
    bias_h = np.ascontiguousarray(np.broadcast_to(full[:, :, :, :S], (B, H, S, S)))
    o_ref, lse_ref = oracle_lib.attention(q, k, v, True, 1 / math.sqrt(D), 1, bias=bias_h)
    dfull = to_dev(full, "bf16").view(1, H, S, S + 3)
    dbias = dfull[:, :, :, :S].expand(B, H, S, S)      # batch stride 0, row stride S + 3
    dq, dk, dv = _dev4(q, "bf16"), _dev4(k, "bf16"), _dev4(v, "bf16")
    do = torch.empty_like(dq)
    dl = torch.empty(B, H, S, dtype=torch.float32, device=cuda)
    assert zlift_b200.fmha_forward(dq, dk, dv, do, dl, mask_type=2, bias=dbias) == 0
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    got = as_float(from_dev(do.reshape(-1), "bf16").reshape(q.shape), "bf16")
    assert normwise(got, as_float(o_ref, "bf16")) <= O_TOL
    assert np.max(np.abs(dl.cpu().numpy() - lse_ref)) <= LSE_TOL


@pytest.mark.parametrize("chunk", ["1", "3", "5", "64"])
def test_flash_block_order_chunks(oracle_lib, cuda, chunk, monkeypatch):
    """The block -> (batch, head, query-tile pair) order in chunks of heads
    (ZBLAS_FMHA_CHUNK; the default depends on the K/V size): every pair is
    computed exactly once for chunk sizes that divide the 2 x 7 heads, leave
    a partial last chunk, or exceed them; outputs start as NaN, so a pair
    that was skipped or written twice with another's data fails."""
    monkeypatch.setenv("ZBLAS_FMHA_CHUNK", chunk)
    run_flash(oracle_lib, "bf16", 2, 640, 640, 7, 7, 128, True, seed=31)


@pytest.mark.parametrize("chunk", ["2", "16"])
def test_flash_pair_range_chunks(oracle_lib, cuda, chunk, monkeypatch):
    """A (batch, head) sub-range (what one rank of a split runs) in chunks:
    the pairs of the range are computed, the rest of O is left untouched."""
    import torch
    import zlift_b200
    from zlift_b200 import attention, partition, blas
    monkeypatch.setenv("ZBLAS_FMHA_CHUNK", chunk)
    B, S, H, D = 2, 512, 5, 128
    q, k, v = _qkv("bf16", B, S, S, H, H, D, 41)
    o_ref, lse_ref = oracle_lib.attention(q, k, v, True, 1.0 / math.sqrt(D), 1)
    dq, dk, dv = _dev4(q, "bf16"), _dev4(k, "bf16"), _dev4(v, "bf16")
    do = torch.full_like(dq, float("nan"))
    dl = torch.full((B, H, S), float("nan"), dtype=torch.float32, device=dq.device)
    blk = attention.flash_block(dq, dk, dv, do, dl, causal=True)
    lo, hi = 3, 9                      # (batch, head) pairs 3..8: b0 h3-4, b1 h0-3
    assert partition.flash_pairs(blk, 1, lo, hi) == 0
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    o = as_float(from_dev(do.reshape(-1), "bf16").reshape(q.shape), "bf16")
    want = as_float(o_ref, "bf16")
    for pair in range(B * H):
        b, h = divmod(pair, H)
        if lo <= pair < hi:
            assert normwise(o[b, :, h], want[b, :, h]) <= O_TOL
        else:
            assert np.all(np.isnan(o[b, :, h]))
