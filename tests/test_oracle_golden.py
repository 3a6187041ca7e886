"""Pin the CPU oracle to the reference: its bytes must equal the fixtures that the
reference's own kquant.py / ef.py produced (tests/golden/make_golden.py)."""
import numpy as np
import pytest

from conftest import K_TYPES

ALL_TYPES = K_TYPES + ["Q8_0"]


@pytest.mark.parametrize("case", ["t3", "cubic", "edge"])
@pytest.mark.parametrize("qmode", ["imat", "imat0", "ref"])
@pytest.mark.parametrize("tt", ALL_TYPES)
def test_oracle_quantize_matches_reference_bytes(orc, kq_golden, case, qmode, tt):
    x = kq_golden[f"x/{case}"]
    qw = None if qmode == "ref" else kq_golden["qw" if qmode == "imat" else "qw0"]
    got = orc.quantize(tt, x, qw)
    want = kq_golden[f"raw/{case}/{qmode}/{tt}"]
    assert got.shape == want.shape
    assert np.array_equal(got, want), f"{np.count_nonzero(got != want)} bytes differ"


@pytest.mark.parametrize("qmode", ["imat", "imat0", "ref"])
@pytest.mark.parametrize("tt", ALL_TYPES)
def test_oracle_dequantize_matches_reference(orc, kq_golden, qmode, tt):
    raw = kq_golden[f"raw/t3/{qmode}/{tt}"]
    want = kq_golden[f"deq/t3/{qmode}/{tt}"]
    got = orc.dequantize(tt, raw, want.shape[1])
    assert np.array_equal(got.view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("tt", K_TYPES)
def test_oracle_repack_of_own_codes_is_identity(orc, kq_golden, tt):
    raw = kq_golden[f"raw/cubic/imat/{tt}"]
    nrow, n = 8, 1024
    L = orc.codes(tt, raw, nrow, n)
    assert np.array_equal(orc.repack(tt, raw, L, nrow, n), raw)


def test_oracle_factor_matches_reference(orc, ef_golden, factor_golden):
    H = ef_golden["H"].astype(np.float64)
    order = ef_golden["order"]
    assert np.array_equal(np.argsort(-np.diag(H)), order)
    U = orc.cholesky_inv_upper(H[np.ix_(order, order)], 0.01).astype(np.float32)
    iu = np.triu_indices(H.shape[0])
    assert np.array_equal(U[iu], ef_golden["U_upper"])
    # escalation path (one negative eigenvalue) and the well-conditioned path, bit for bit
    assert np.array_equal(orc.cholesky_inv_upper(factor_golden["H_bad"]), factor_golden["U_bad"])
    assert np.array_equal(orc.cholesky_inv_upper(factor_golden["H_pd"]), factor_golden["U_pd"])


@pytest.mark.parametrize("qmode", ["imat", "ref"])
@pytest.mark.parametrize("tt", K_TYPES)
def test_oracle_ef_matches_reference_bytes(orc, ef_golden, tt, qmode):
    W = ef_golden[f"W/{tt}"]
    H = ef_golden["H"].astype(np.float64)
    qw = ef_golden["qw"] if qmode == "imat" else None
    raw, recon = orc.ef_encode(W, tt, qw, H, n_iter=2, act_order=True)
    assert np.array_equal(raw, ef_golden[f"raw/{qmode}/{tt}"])
    assert np.array_equal(recon.view(np.int32), ef_golden[f"recon/{qmode}/{tt}"].view(np.int32))


@pytest.mark.parametrize("tt", K_TYPES)
def test_oracle_ef_single_iteration_and_storage_order(orc, ef_golden, tt):
    W = ef_golden[f"W/{tt}"]
    H = ef_golden["H"].astype(np.float64)
    qw = ef_golden["qw"]
    raw1, _ = orc.ef_encode(W, tt, qw, H, n_iter=1, act_order=True)
    assert np.array_equal(raw1, ef_golden[f"raw1/imat/{tt}"])
    raws, _ = orc.ef_encode(W, tt, qw, H, n_iter=2, act_order=False)
    assert np.array_equal(raws, ef_golden[f"raw_storage/imat/{tt}"])
