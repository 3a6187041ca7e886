"""perm_b200.objective.tensor_err / col_log_rms against the reference formula
(coldpress/perm/objective.py:17-51) restated here with the oracle's k-quant roundtrip."""
import zlib

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _ref_tensor_err(orc, x, ttype, qw, perm=None, wvec=None, rows_sample=None, seed=0):
    if rows_sample and x.shape[0] > rows_sample:
        rng = np.random.default_rng(seed)
        idx = np.sort(rng.choice(x.shape[0], rows_sample, replace=False))
        x = x[idx]
    x = np.asarray(x, dtype=np.float32)
    if perm is not None:
        x = x[:, perm]
        qw = qw[perm] if qw is not None else None
    recon = orc.roundtrip(np.ascontiguousarray(x), ttype, qw)
    colerr = ((recon.astype(np.float64) - x.astype(np.float64)) ** 2).sum(0)
    if wvec is not None:
        w = wvec[perm] if perm is not None else wvec
        return float((colerr * w).sum())
    if qw is not None:
        return float((colerr * qw).sum())
    return float(colerr.sum())


@pytest.mark.parametrize("ttype", ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"])
@pytest.mark.parametrize("case", ["plain", "perm", "perm_wvec", "sample", "no_qw"])
def test_tensor_err_matches_reference_formula(orc, ttype, case):
    from perm_b200 import objective
    rng = np.random.default_rng(zlib.crc32(f"{ttype}/{case}".encode()))
    x = (rng.standard_normal((96, 512)) * rng.lognormal(0, 1, 512) * 0.02).astype(np.float32)
    qw = rng.lognormal(0, 1, 512).astype(np.float32)
    kw = {}
    if case in ("perm", "perm_wvec"):
        kw["perm"] = rng.permutation(512)
    if case == "perm_wvec":
        kw["wvec"] = rng.lognormal(0, 1, 512)
    if case == "sample":
        kw["rows_sample"], kw["seed"] = 40, 7
    if case == "no_qw":
        qw = None
    want = _ref_tensor_err(orc, x, ttype, qw, **kw)
    got = objective.tensor_err(x, ttype, qw, **kw)
    assert got == pytest.approx(want, rel=1e-12)


def test_tensor_err_float_types_and_torch_inputs(orc):
    import torch
    from perm_b200 import objective
    rng = np.random.default_rng(5)
    x = (rng.standard_normal((64, 256)) * 0.02).astype(np.float32)
    qw = rng.lognormal(0, 1, 256).astype(np.float32)
    for t in ("F16", "F32", "BF16"):
        assert objective.tensor_err(x, t, qw) == 0.0
    perm = rng.permutation(256)
    want = _ref_tensor_err(orc, x, "Q2_K", qw, perm=perm)
    got = objective.tensor_err(torch.from_numpy(x).cuda(), "Q2_K", torch.from_numpy(qw).cuda(),
                               perm=torch.from_numpy(perm).cuda())
    assert got == pytest.approx(want, rel=1e-12)
    with pytest.raises(ValueError):
        objective.tensor_err(x, "Q8_K", qw)


def test_col_log_rms_matches_reference_formula():
    from perm_b200 import objective
    rng = np.random.default_rng(11)
    x = (rng.standard_normal((1000, 256)) * 0.02).astype(np.float32)
    acc = np.zeros(256, np.float64)
    for r0 in range(0, 1000, 300):
        xc = np.asarray(x[r0:r0 + 300], dtype=np.float64)
        acc += (xc ** 2).sum(0)
    want = np.log(np.sqrt(acc / 1000) + 1e-12)
    np.testing.assert_allclose(objective.col_log_rms(x, row_step=300), want, rtol=1e-13, atol=0)
