"""Parity at BASELINE config sizes against the reference's OWN outputs
(tests/golden/config_golden.npz, written by tests/golden/make_golden_config.py, which runs the
reference's kquant.QUANTIZE and ef.ef_encode on the seeded inputs of
tests/golden/config_inputs.py):

  * config[1]: 4096 x 4096 plain k-quant, 5 types x {imatrix, reference path}: the SHA-256
    of the CUDA path's bytes (and of the CPU oracle's) equals the reference's;
  * config[0]: 3072 x 1024 EF Q2_K: the CUDA path's bytes equal the reference's (codes and
    H-weighted-error gates asserted first, then byte identity).

Each test first proves it rebuilt the very inputs the reference saw (their SHA-256)."""
import os
import sys

import numpy as np
import pytest

from conftest import GOLDEN, K_TYPES, h_weighted_err

sys.path.insert(0, GOLDEN)
import config_inputs as ci  # noqa: E402


@pytest.fixture(scope="module")
def golden():
    return dict(np.load(os.path.join(GOLDEN, "config_golden.npz")))


@pytest.fixture(scope="module")
def c1(golden):
    W, qw = ci.config1()
    assert ci.sha(W) == str(golden["c1_W_sha"]) and ci.sha(qw) == str(golden["c1_qw_sha"]), \
        "config[1] inputs differ from the ones the reference encoded"
    return W, qw


@pytest.fixture(scope="module")
def c0(golden):
    W, H, qw = ci.config0()
    assert ci.sha(W) == str(golden["c0_W_sha"]) and ci.sha(H) == str(golden["c0_H_sha"]), \
        "config[0] inputs differ from the ones the reference encoded"
    return W, H, qw


@pytest.mark.parametrize("tt", K_TYPES)
def test_oracle_matches_reference_at_config1(golden, c1, orc, tt):
    W, qw = c1
    for path, q in (("imat", qw), ("ref", None)):
        raw = orc.quantize(tt, W, q)
        assert ci.sha(raw) == str(golden[f"c1_{tt}_{path}_sha"]), f"oracle {tt} {path}"


def test_oracle_matches_reference_at_config0(golden, c0, orc):
    W, H, qw = c0
    raw, _ = orc.ef_encode(W, "Q2_K", qw, H, n_iter=2, act_order=True)
    want = golden["c0_raw"]
    frac = float(np.mean(orc.codes("Q2_K", raw, *W.shape) == orc.codes("Q2_K", want, *W.shape)))
    print(f"oracle config0 EF vs reference: codes identical {frac:.5%}, bytes identical {np.array_equal(raw, want)}")
    assert frac >= 0.999


@pytest.mark.gpu
@pytest.mark.parametrize("tt", K_TYPES)
@pytest.mark.parametrize("path", ["imat", "ref"])
def test_cuda_matches_reference_at_config1(golden, c1, tt, path):
    from perm_b200 import kquant
    W, qw = c1
    raw = kquant.QUANTIZE[tt](W, qw if path == "imat" else None)
    assert tuple(raw.shape) == tuple(golden[f"c1_{tt}_{path}_shape"])
    assert ci.sha(raw) == str(golden[f"c1_{tt}_{path}_sha"]), f"{tt} {path}: bytes differ from the reference"


@pytest.mark.gpu
def test_cuda_ef_matches_reference_at_config0(golden, c0, orc):
    from perm_b200 import ef
    W, H, qw = c0
    raw, recon = ef.ef_encode(W, "Q2_K", qw, H, n_iter=2, act_order=True)
    want = golden["c0_raw"]
    frac = float(np.mean(orc.codes("Q2_K", raw, *W.shape) == orc.codes("Q2_K", want, *W.shape)))
    rel = h_weighted_err(W, recon, H) / h_weighted_err(W, orc.dequantize("Q2_K", want, W.shape[1]), H) - 1
    print(f"CUDA config0 EF vs reference: codes identical {frac:.5%}, H-err rel {rel:+.2e}, "
          f"bytes identical {np.array_equal(raw, want)}")
    assert frac >= 0.999 and abs(rel) <= 1e-3
    assert np.array_equal(raw, want), f"{np.count_nonzero(raw != want)} bytes differ from the reference"
