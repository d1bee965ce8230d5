"""Shared fixtures for the rouge-numerics-b200 tests.

CPU tests (no mark) check the oracle against the reference's golden vectors,
the host logic and the C ABI surface. GPU tests are marked `gpu` and compare
the sm_100a kernels, called through the C ABI, with the oracle.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "rouge-v_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))
GOLDEN = os.path.join(ROOT, "tests", "golden", "golden.npz")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs an sm_100 (B200) GPU")


def _ensure_built():
    import oracle as O
    import rouge_b200 as rb
    if not os.path.exists(O.ORACLE_SO) or not os.path.exists(rb.LIB_PATH):
        sys.path.insert(0, ROOT)
        import __graft_entry__
        __graft_entry__.build()


@pytest.fixture(scope="session")
def orc():
    _ensure_built()
    import oracle as O
    return O.Oracle()


@pytest.fixture(scope="session")
def ref():
    import oracle as O
    if not O.Reference.available():
        pytest.skip("reference library oracle/_ref/librouge_ref.so not built")
    return O.Reference()


@pytest.fixture(scope="session")
def rb():
    _ensure_built()
    import rouge_b200
    rouge_b200.lib()
    return rouge_b200


@pytest.fixture(scope="session")
def golden():
    return dict(np.load(GOLDEN))


@pytest.fixture(scope="session")
def cuda(rb):
    import torch
    if not torch.cuda.is_available():
        pytest.fail("GPU test run without a CUDA device")
    assert rb.lib().rouge_b200_device_ok() == 1, "device is not an sm_100 part"
    return torch.device("cuda:0")


def rel_l2(got, want) -> float:
    got = np.asarray(got, np.float64)
    want = np.asarray(want, np.float64)
    return float(np.linalg.norm(got - want) / max(np.linalg.norm(want), 1e-300))
