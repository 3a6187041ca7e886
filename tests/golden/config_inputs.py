"""Seeded inputs of BASELINE config[0] and config[1], shared by make_golden_config.py (which
runs the reference on them) and the tests (which run the CUDA path and check, by SHA-256,
that they rebuilt the very same inputs)."""
import hashlib

import numpy as np

K_TYPES = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def sha(a):
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def config1(seed=20261202):
    """4096 x 4096 float32 weights 0.02 * Student-t(3), imatrix log-normal(0, 1) per column."""
    rng = np.random.default_rng(seed)
    W = (0.02 * rng.standard_t(3, size=(4096, 4096))).astype(np.float32)
    qw = rng.lognormal(0.0, 1.0, 4096).astype(np.float32)
    return W, qw


def config0(seed=20261203):
    """3072 x 1024 float32 weights N(0, 0.02) with 1 % of the input columns x8; H = X^T X / 8192
    (float64) for X = N(0, 1) x per-channel log-normal(0, 1); qw = diag(H).  X is drawn on a
    grid of 1/16 so that X^T X is an exact integer sum (below 2^53) whatever order a BLAS adds
    it in: H comes out bit-identical on every machine."""
    rng = np.random.default_rng(seed)
    W = (rng.standard_normal((3072, 1024)) * 0.02).astype(np.float32)
    W[:, rng.choice(1024, 10, replace=False)] *= 8.0
    Xq = np.round(rng.standard_normal((8192, 1024)) * 16.0)   # integers: X = Xq / 16
    s = rng.lognormal(0.0, 1.0, 1024)
    H = (Xq.T @ Xq) * np.outer(s, s) / (256.0 * 8192)
    return W, H, np.diag(H).astype(np.float32)
