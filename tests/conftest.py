"""Shared test setup.

Markers: `gpu` tests need a CUDA device (a B200); everything else runs on the CPU.
The CPU oracle (oracle/kquant_oracle.c) is compiled on first use.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

GOLDEN = os.path.join(ROOT, "tests", "golden")
K_TYPES = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200, sm_100a)")


@pytest.fixture(scope="session")
def orc():
    from oracle import oracle
    oracle.build()
    return oracle


@pytest.fixture(scope="session")
def kq_golden():
    return dict(np.load(os.path.join(GOLDEN, "kquant_golden.npz")))


@pytest.fixture(scope="session")
def ef_golden():
    return dict(np.load(os.path.join(GOLDEN, "ef_golden.npz")))


@pytest.fixture(scope="session")
def factor_golden():
    return dict(np.load(os.path.join(GOLDEN, "factor_golden.npz")))


def heavy_tailed(nrow, n, seed):
    """Heavy-tailed weights: N(0,1)^3 times a per-row U(0.2, 3) scale."""
    rng = np.random.default_rng(seed)
    x = (rng.standard_normal((nrow, n)) ** 3).astype(np.float32)
    x *= rng.uniform(0.2, 3.0, size=(nrow, 1)).astype(np.float32)
    return x


def h_weighted_err(W, What, H):
    D = (What - W).astype(np.float64)
    return float(np.einsum("ri,ij,rj->", D, H, D))
