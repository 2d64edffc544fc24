"""Shared fixtures.  `-m gpu` tests need a B200; everything else runs on CPU.

The oracle (oracle/liboracle.so, and oracle/_ref/libzblas_ref.so where the
reference tree exists) and the product library are built on first use if
they are missing."""
import os
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

# PyTorch first: its cuBLAS/cuDNN must be the ones the loader binds for it,
# before anything in this process could load this repository's drop-in
# libraries (which carry the cuBLAS 13 / cuDNN 9 sonames).
import torch  # noqa: E402,F401


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an NVIDIA B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def built_lib():
    import zlift_b200
    from zlift_b200 import build
    if not os.path.exists(zlift_b200.LIBCUBLAS):
        build.build()
    return zlift_b200.load()


@pytest.fixture(scope="session")
def oracle_lib():
    from oracle import oracle
    if not os.path.exists(oracle.ORACLE_SO):
        oracle.build(ref=True)
    return oracle


@pytest.fixture(scope="session")
def cuda(built_lib):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.init()
    return torch.device("cuda:0")
