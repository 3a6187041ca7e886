"""CUDA k-quant codec vs the reference: byte-identical output.

Small cases compare with the reference's own bytes (tests/golden); the 4096x4096
configuration (bit-exactness sweep over all types, imatrix and reference paths) compares
with the CPU oracle, which is itself pinned to the reference."""
import numpy as np
import pytest

from conftest import K_TYPES

pytestmark = pytest.mark.gpu
ALL_TYPES = K_TYPES + ["Q8_0"]


@pytest.fixture(scope="module")
def kq():
    from perm_b200 import kquant
    return kquant


@pytest.mark.parametrize("case", ["t3", "cubic", "edge"])
@pytest.mark.parametrize("qmode", ["imat", "imat0", "ref"])
@pytest.mark.parametrize("tt", ALL_TYPES)
def test_quantize_matches_reference_golden(kq, kq_golden, case, qmode, tt):
    x = kq_golden[f"x/{case}"]
    qw = None if qmode == "ref" else kq_golden["qw" if qmode == "imat" else "qw0"]
    got = kq.QUANTIZE[tt](x, qw)
    want = kq_golden[f"raw/{case}/{qmode}/{tt}"]
    assert got.dtype == np.uint8 and got.shape == want.shape
    bad = np.count_nonzero(got != want)
    assert bad == 0, f"{bad} bytes differ"


@pytest.mark.parametrize("qmode", ["imat", "ref"])
@pytest.mark.parametrize("tt", ALL_TYPES)
def test_dequantize_matches_reference_golden(kq, kq_golden, qmode, tt):
    raw = kq_golden[f"raw/t3/{qmode}/{tt}"]
    want = kq_golden[f"deq/t3/{qmode}/{tt}"]
    got = kq.DEQUANTIZE[tt](raw, want.shape[1])
    assert np.array_equal(got.view(np.int32), want.view(np.int32))


@pytest.mark.parametrize("qmode", ["imat", "ref"])
@pytest.mark.parametrize("tt", K_TYPES)
def test_quantize_4096x4096_matches_oracle(kq, orc, tt, qmode):
    rng = np.random.default_rng(1)
    x = (rng.standard_t(3, size=(4096, 4096)) * 0.02).astype(np.float32)
    qw = rng.lognormal(0.0, 1.0, 4096).astype(np.float32) if qmode == "imat" else None
    got = kq.QUANTIZE[tt](x, qw)
    want = orc.quantize(tt, x, qw)
    bb = orc.BYTES_PER_BLOCK[tt]
    bad_blocks = np.count_nonzero((got.reshape(-1, bb) != want.reshape(-1, bb)).any(1))
    assert bad_blocks == 0, f"{bad_blocks} of {want.size // bb} superblocks differ"


@pytest.mark.parametrize("tt", K_TYPES)
def test_ragged_rows_and_single_superblock(kq, orc, tt):
    rng = np.random.default_rng(5)
    for nrow, n in ((1, 256), (3, 512), (17, 768), (33, 256)):
        x = (rng.standard_normal((nrow, n)) ** 3).astype(np.float32)
        qw = rng.lognormal(0.0, 1.0, n).astype(np.float32)
        for q in (qw, None):
            assert np.array_equal(kq.QUANTIZE[tt](x, q), orc.quantize(tt, x, q)), (nrow, n)


def test_empty_and_bad_shapes(kq):
    x = np.zeros((0, 512), np.float32)
    assert kq.QUANTIZE["Q4_K"](x, None).shape == (0, 2 * 144)
    with pytest.raises(AssertionError):
        kq.QUANTIZE["Q2_K"](np.zeros((2, 200), np.float32), None)
    with pytest.raises(ValueError):
        kq.QUANTIZE["Q4_K"](np.zeros((2, 200), np.float32), None)
    with pytest.raises(KeyError):  # an unknown type is a missing dict key, as in kquant.py:732
        kq.QUANTIZE["Q9_K"]


@pytest.mark.parametrize("tt", K_TYPES)
def test_grid_codes_repack_roundtrip(kq, orc, kq_golden, tt):
    import torch
    raw = kq_golden[f"raw/cubic/imat/{tt}"]
    nrow, n = 8, 1024
    rd = torch.from_numpy(raw).cuda()
    dl, ml, lo, hi, sbw = kq.grid_params_dev(tt, rd, nrow, n)
    odl, oml = orc.grid_params(tt, raw, nrow, n)
    assert np.array_equal(dl.cpu().numpy(), odl)
    if ml is not None:
        assert np.array_equal(ml.cpu().numpy(), oml)
    c = kq.codes_dev(tt, rd, nrow, n)
    assert np.array_equal(c.cpu().numpy().astype(np.int32), orc.codes(tt, raw, nrow, n))
    scrambled = rd.clone()
    off = {"Q2_K": (16, 80), "Q3_K": (0, 96), "Q4_K": (16, 144), "Q5_K": (16, 176), "Q6_K": (0, 192)}[tt]
    scrambled.view(-1, orc.BYTES_PER_BLOCK[tt])[:, off[0]:off[1]] = 0
    kq.repack_dev(tt, scrambled, c, nrow, n)
    assert np.array_equal(scrambled.cpu().numpy(), raw)
