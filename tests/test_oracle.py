"""CPU: pins the oracle (the C restatement in oracle/zlift_oracle.c).

1. Against the committed golden vectors in tests/golden/, which were made
   by running the reference's own zblas.c CPU path (tests/golden/make_golden.py).
2. Against the reference library itself (oracle/_ref/libzblas_ref.so, built
   from the reference sources) on fresh seeded inputs, where it exists.
3. The converters against the reference converters' contract: fp16 rounds
   to nearest-even for normals and truncates subnormals; bf16 rounds to
   nearest-even.
"""
import json
import os

import numpy as np
import pytest

from tests.helpers import as_float, normwise

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load_golden():
    with open(os.path.join(GOLDEN, "gemm_cases.json")) as f:
        return json.load(f)


def _arr(case, name):
    meta = case[name]
    raw = np.load(os.path.join(GOLDEN, case["file"]))[name]
    return raw.astype(np.dtype(meta))


@pytest.mark.parametrize("idx", range(len(_load_golden()["cases"])))
def test_oracle_matches_reference_golden(oracle_lib, idx):
    """The restatement reproduces the reference CPU path's stored outputs."""
    case = _load_golden()["cases"][idx]
    data = np.load(os.path.join(GOLDEN, case["file"]))
    A, B, C0, want = data["A"], data["B"], data["C0"], data["C"]
    C = C0.copy()
    rc = oracle_lib.gemm_ex(case["ta"], case["tb"], case["m"], case["n"], case["k"],
                            case["alpha"], A, case["Atype"], case["lda"], B, case["Btype"],
                            case["ldb"], case["beta"], C, case["Ctype"], case["ldc"],
                            case["compute"])
    if case["Atype"] == 3:
        # the reference answers int8 with NOT_SUPPORTED (zblas.c:366-367); the
        # restatement's int8 branch is new and is pinned by test_int8_oracle_exact
        assert case["status"] == 15 and rc == 0
        return
    assert rc == case["status"]
    if rc != 0:
        return
    ck = {0: "f32", 2: "f16", 14: "bf16", 10: "i32"}[case["Ctype"]]
    if ck == "i32":
        np.testing.assert_array_equal(C, want)
        return
    got, ref = as_float(C, ck), as_float(want, ck)
    tol = 1e-6 if ck == "f32" else 8e-3
    assert normwise(got, ref) <= tol
    # narrow outputs: all but a few elements are bit-identical (the two sides
    # sum in different orders, so an element can land on a neighbour)
    if ck != "f32":
        assert np.mean(C != want) < 0.02


def test_golden_cover_all_configs():
    cases = _load_golden()["cases"]
    kinds = {(c["Atype"], c["Ctype"]) for c in cases}
    assert (0, 0) in kinds and (2, 2) in kinds and (14, 14) in kinds
    assert any(c["status"] == 15 for c in cases)   # int8 is NOT_SUPPORTED in the reference


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__))), "oracle", "_ref", "libzblas_ref.so")),
    reason="reference library not built here")
@pytest.mark.parametrize("kind,ta,tb,m,n,k,alpha,beta", [
    ("f16", 0, 1, 64, 48, 80, 1.0, 0.5),
    ("bf16", 0, 0, 33, 65, 17, 0.3, 0.0),
    ("f32", 1, 1, 40, 30, 50, -1.0, 2.0),
    ("f16", 1, 0, 128, 16, 256, 2.0, -0.5),
])
def test_oracle_matches_reference_live(oracle_lib, kind, ta, tb, m, n, k, alpha, beta):
    from zlift_b200 import inputs
    T = {"f16": 2, "bf16": 14, "f32": 0}[kind]
    ar, ac = (m, k) if ta == 0 else (k, m)
    br, bc = (k, n) if tb == 0 else (n, k)
    A = inputs.make(kind, "normal", 11, ar * ac)
    B = inputs.make(kind, "normal", 12, br * bc)
    C0 = inputs.make(kind, "normal", 13, m * n)
    c1, c2 = C0.copy(), C0.copy()
    if kind == "f32":
        rc1 = oracle_lib.ref_sgemm(ta, tb, m, n, k, alpha, A, ar, B, br, beta, c1, m)
    else:
        rc1 = oracle_lib.ref_gemm_ex(ta, tb, m, n, k, alpha, A, T, ar, B, T, br, beta, c1, T, m)
    rc2 = oracle_lib.gemm_ex(ta, tb, m, n, k, alpha, A, T, ar, B, T, br, beta, c2, T, m)
    assert rc1 == rc2 == 0
    assert normwise(as_float(c2, kind), as_float(c1, kind)) <= (1e-6 if kind == "f32" else 8e-3)


@pytest.mark.skipif(not os.path.exists(os.path.join(os.path.dirname(os.path.dirname(
    os.path.abspath(__file__))), "oracle", "_ref", "libzblas_ref.so")),
    reason="reference library not built here")
def test_reference_rejects_int8(oracle_lib):
    """The reference has no int8 GEMM: status 15 for compute 32I and 32F."""
    A = np.ones(64, dtype=np.int8)
    C = np.zeros(64, dtype=np.int32)
    for compute in (72, 68):
        assert oracle_lib.ref_gemm_ex(0, 0, 8, 8, 8, 1, A, 3, 8, A, 3, 8, 0, C, 10, 8,
                                      compute) == 15


def test_int8_oracle_exact(oracle_lib):
    from zlift_b200 import inputs
    m, n, k = 17, 23, 300
    A = inputs.int8(1, k * m)
    B = inputs.int8(2, k * n)
    C = np.zeros(m * n, dtype=np.int32)
    assert oracle_lib.gemm_ex(1, 0, m, n, k, 1, A, 3, k, B, 3, k, 0, C, 10, m, 72) == 0
    want = (A.reshape(m, k).astype(np.int64) @ B.reshape(n, k).astype(np.int64).T)
    np.testing.assert_array_equal(C.reshape(n, m), want.T.astype(np.int32))


def test_converters(oracle_lib):
    # every fp16 bit pattern widens like numpy's float16 (NaN payloads aside)
    bits = np.arange(65536, dtype=np.uint16)
    f = oracle_lib.half_to_float(bits)
    ref = bits.view(np.float16).astype(np.float32)
    finite = np.isfinite(ref)
    np.testing.assert_array_equal(f[finite], ref[finite])
    # normals narrow with round-to-nearest-even
    x = np.array([1.0, 1.0 + 2 ** -11, 1.0 + 3 * 2 ** -11, 65504.0, 7e4, -2.5], np.float32)
    np.testing.assert_array_equal(oracle_lib.float_to_half(x),
                                  np.array([0x3C00, 0x3C00, 0x3C02, 0x7BFF, 0x7C00, 0xC100],
                                           np.uint16))
    # subnormals truncate (reference zblas.c:268-272): 1.9 * 2^-24 -> 0x0001
    assert oracle_lib.float_to_half(np.array([1.9 * 2 ** -24], np.float32))[0] == 1
    # bf16: round to nearest even on the low 16 bits
    u = np.array([0x3F808000, 0x3F818000, 0x3F80C000], np.uint32).view(np.float32)
    np.testing.assert_array_equal(oracle_lib.float_to_bf16(u),
                                  np.array([0x3F80, 0x3F82, 0x3F81], np.uint16))
    b = np.array([0x3F80, 0xC2F7], np.uint16)
    np.testing.assert_array_equal(oracle_lib.bf16_to_float(b), np.array([1.0, -123.5], np.float32))


def test_attention_oracle_small(oracle_lib):
    """Attention restatement against a direct numpy evaluation (fp32 inputs,
    where no rounding of P applies)."""
    from zlift_b200 import inputs
    B, S, H, D = 1, 9, 2, 16
    q = inputs.normal(1, B * S * H * D).astype(np.float32).reshape(B, S, H, D)
    k = inputs.normal(2, B * S * H * D).astype(np.float32).reshape(B, S, H, D)
    v = inputs.normal(3, B * S * H * D).astype(np.float32).reshape(B, S, H, D)
    scale = 0.25
    for causal in (False, True):
        o, lse = oracle_lib.attention(q, k, v, causal, scale, elem=2)
        for h in range(H):
            s = (q[0, :, h, :].astype(np.float64) @ k[0, :, h, :].astype(np.float64).T) * scale
            if causal:
                s[np.triu_indices(S, 1)] = -np.inf
            mx = s.max(axis=1, keepdims=True)
            p = np.exp(s - mx)
            l = p.sum(axis=1, keepdims=True)
            want = (p / l) @ v[0, :, h, :].astype(np.float64)
            np.testing.assert_allclose(o[0, :, h, :], want, rtol=2e-6, atol=2e-6)
            np.testing.assert_allclose(lse[0, h], (mx + np.log(l))[:, 0], rtol=1e-6)


def test_attention_oracle_masked_rows(oracle_lib):
    """Causal with Sq > Sk, bottom-right aligned: the first Sq-Sk query rows
    see no key; O is 0 there (zblas_gpu.cpp:981, :991, :1015)."""
    from zlift_b200 import inputs
    B, Sq, Sk, H, D = 1, 6, 3, 1, 16
    q = inputs.make("bf16", "normal", 1, B * Sq * H * D).reshape(B, Sq, H, D)
    k = inputs.make("bf16", "normal", 2, B * Sk * H * D).reshape(B, Sk, H, D)
    v = inputs.make("bf16", "normal", 3, B * Sk * H * D).reshape(B, Sk, H, D)
    o, lse = oracle_lib.attention(q, k, v, True, 0.25, elem=1)
    assert np.all(o[0, :3] == 0)
    assert np.all(np.isneginf(lse[0, 0, :3]))
    assert np.all(np.isfinite(lse[0, 0, 3:]))
