"""Fused attention forward parity on the GPU, through the C ABI
(zlift_flash_fwd / zlift_fmha_fwd in libcublas.so.13), against the oracle's
restatement of the reference attention math (fmha_f32 / fmha_run).

Tolerances: O normwise (max|x - ref| / max|ref|) <= 1e-2; LSE absolute
<= 1e-3 (LSE is about log(S) ~ 8, so this is ~1e-4 relative).  The
reference never produces LSE, so the LSE checks pin it against the
restatement only.
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


def run_flash(oracle, kind, B, Sq, Sk, H, Hk, D, causal, seed=1, api="flash"):
    import torch
    import zlift_b200
    from zlift_b200 import blas
    q, k, v = _qkv(kind, B, Sq, Sk, H, Hk, D, seed)
    scale = 1.0 / math.sqrt(D)
    elem = 1 if kind == "bf16" else 0
    o_ref, lse_ref = oracle.attention(q, k, v, causal, scale, elem, kv_ratio=H // Hk)
    dq, dk, dv = _dev4(q, kind), _dev4(k, kind), _dev4(v, kind)
    do = torch.full_like(dq, float("nan"))
    dl = torch.full((B, H, Sq), float("nan"), dtype=torch.float32, device=dq.device)
    if api == "flash":
        rc = zlift_b200.flash_forward(dq, dk, dv, do, dl, causal=causal, scale=scale)
    else:
        rc = zlift_b200.fmha_forward(dq, dk, dv, do, dl, mask_type=2 if causal else 0,
                                     scale=scale)
    assert rc == 0, f"entry returned {rc}"
    torch.cuda.synchronize()
    assert blas.device_error() == 0
    o = from_dev(do.reshape(-1), kind).reshape(q.shape)
    got, want = as_float(o, kind), as_float(o_ref, kind)
    assert np.all(np.isfinite(got))
    err = normwise(got, want)
    assert err <= O_TOL, f"O normwise error {err:.3e}"
    lse = dl.cpu().numpy()
    fin = np.isfinite(lse_ref)
    np.testing.assert_array_equal(np.isfinite(lse), fin)
    if fin.any():
        assert np.max(np.abs(lse[fin] - lse_ref[fin])) <= LSE_TOL
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
