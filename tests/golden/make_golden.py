"""Generates the golden GEMM vectors in this folder by running the
reference's own CPU path -- zLift's zblas/zblas.c compiled unmodified into
oracle/_ref/libzblas_ref.so by oracle/Makefile (`make -C oracle ref`) --
on small seeded inputs shaped like each benchmark configuration.

Run from the repository root where the reference tree is present:
    python tests/golden/make_golden.py
Outputs gemm_cases.json (the case list) and one .npz per case (inputs A,
B, C0 and the reference's output C).
"""
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)

from oracle import oracle  # noqa: E402
from zlift_b200 import inputs  # noqa: E402

# (name, kind, ta, tb, m, n, k, alpha, beta, Ctype, compute)
CASES = [
    # configuration 1 shape family: fp32 NN, alpha 1 beta 0, uniform inputs
    ("sgemm_nn", "f32", 0, 0, 48, 40, 56, 1.0, 0.0, 0, 68),
    ("sgemm_tt_ab", "f32", 1, 1, 33, 29, 47, -0.5, 1.5, 0, 0),
    # configuration 2 family: fp16 NT, beta 0.5, fp16 out
    ("gemmex_f16_nt", "f16", 0, 1, 64, 48, 64, 1.0, 0.5, 2, 68),
    ("gemmex_f16_tn_f32out", "f16", 1, 0, 40, 24, 72, 0.75, 0.0, 0, 68),
    # configuration 3 family: bf16 NN, alpha 1/sqrt(k)
    ("gemmex_bf16_nn", "bf16", 0, 0, 32, 48, 64, 1.0 / 8.0, 0.0, 14, 68),
    ("gemmex_bf16_nt_f32out", "bf16", 0, 1, 24, 16, 40, 1.0, 1.0, 0, 0),
    # configuration 4 family: int8 -> int32 (the reference answers NOT_SUPPORTED)
    ("gemmex_i8_tn", "i8", 1, 0, 16, 16, 32, 1, 0, 10, 72),
]

T = {"f32": 0, "f16": 2, "bf16": 14, "i8": 3}


def main():
    oracle.build(ref=True)
    out = {"generator": "tests/golden/make_golden.py",
           "reference": "zblas/zblas.c CPU path (cblas via numpy's OpenBLAS)", "cases": []}
    for i, (name, kind, ta, tb, m, n, k, alpha, beta, ct, compute) in enumerate(CASES):
        ar, ac = (m, k) if ta == 0 else (k, m)
        br, bc = (k, n) if tb == 0 else (n, k)
        dist = "int8" if kind == "i8" else ("uniform" if kind == "f32" else "normal")
        scale = 1.0 / np.sqrt(k) if kind == "f16" else 1.0
        A = inputs.make(kind, dist, 100 + i, ar * ac, scale)
        B = inputs.make(kind, dist, 200 + i, br * bc, scale)
        ckind = {0: "f32", 2: "f16", 14: "bf16", 10: "i32"}[ct]
        if ckind == "i32":
            C0 = np.zeros(m * n, np.int32)
        else:
            C0 = inputs.make(ckind, "normal", 300 + i, m * n)
        C = C0.copy()
        if kind == "f32":
            rc = oracle.ref_sgemm(ta, tb, m, n, k, alpha, A, ar, B, br, beta, C, m)
        else:
            rc = oracle.ref_gemm_ex(ta, tb, m, n, k, alpha, A, T[kind], ar, B, T[kind], br,
                                    beta, C, ct, m, compute)
        fname = f"{name}.npz"
        np.savez_compressed(os.path.join(HERE, fname), A=A, B=B, C0=C0, C=C)
        out["cases"].append({"name": name, "file": fname, "ta": ta, "tb": tb, "m": m, "n": n,
                             "k": k, "alpha": alpha, "beta": beta, "Atype": T[kind],
                             "Btype": T[kind], "Ctype": ct, "lda": ar, "ldb": br, "ldc": m,
                             "compute": compute, "status": rc})
        print(name, "status", rc)
    with open(os.path.join(HERE, "gemm_cases.json"), "w") as f:
        json.dump(out, f, indent=1)


if __name__ == "__main__":
    main()
