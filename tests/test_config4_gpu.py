"""BASELINE config[4] shapes (Llama-3-8B-shaped, Q4_K_M-style mixture) against the CPU oracle,
a restatement of coldpress/ef.py:46-84 (cholesky_inv_upper) and ef.py:179-218 (ef_encode):

  * the n = 14336 factorisation (ffn_down's input Hessian): the float32 U must equal the
    oracle's on at least 99.9 % of its upper-triangle entries;
  * ffn_down 4096 x 14336 as Q6_K (even layers) and Q4_K (odd layers) and ffn_gate
    14336 x 4096 as Q4_K, encoded whole through the grouped encoder the bench runs
    (Encoder.run); rows sampled across each tensor are re-encoded by the oracle with its own
    U: at least 99.9 % identical codes and an H-weighted error within 0.1 % (the gates of
    the reference's tests, tests/test_ef_synthetic.py), and the bytes themselves are
    reported.

Hessians are H = X^T X / T from T = 32768 synthetic tokens with log-normal channel scales,
formed in float64 on the device (test set-up only)."""
import numpy as np
import pytest

from conftest import h_weighted_err

pytestmark = pytest.mark.gpu

T_TOKENS = 32768


def _hessian(torch, n, seed):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    scales = torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
    H = torch.zeros((n, n), device="cuda", dtype=torch.float64)
    for _ in range(T_TOKENS // 8192):
        X = torch.randn(8192, n, device="cuda", dtype=torch.float64, generator=g) * scales
        H.addmm_(X.T, X)
        del X
    H /= T_TOKENS
    return H


@pytest.fixture(scope="module")
def big():
    import torch
    from perm_b200 import ef
    out = {}
    for n, seed in ((14336, 41), (4096, 42)):
        H = _hessian(torch, n, seed)
        Hh = H.cpu().numpy()
        diag = np.diag(Hh).copy()
        order = np.argsort(-diag)
        U, _ = ef.factor_u_dev(H, order, 0.01, diag_host=diag)
        out[n] = {"H": H, "Hh": Hh, "diag": diag, "order": order, "U_gpu": U.cpu().numpy()}
        torch.cuda.synchronize()
    return out


@pytest.fixture(scope="module")
def oracle_u(big, orc):
    res = {}
    for n, b in big.items():
        Hp = b["Hh"][np.ix_(b["order"], b["order"])]
        res[n] = orc.cholesky_inv_upper(Hp, 0.01).astype(np.float32)
    return res


@pytest.mark.parametrize("n", [14336, 4096])
def test_factor_matches_oracle(big, oracle_u, n):
    got, want = big[n]["U_gpu"], oracle_u[n]
    iu = np.triu_indices(n)
    same = float(np.mean(got[iu] == want[iu]))
    print(f"n={n}: float32 U identical on {same:.5%} of {iu[0].size} entries")
    assert same >= 0.999
    assert np.array_equal(np.tril(got, -1), np.zeros_like(got))


def test_llama_shapes_match_oracle(big, oracle_u, orc):
    import torch
    from perm_b200.encoder import Encoder, Job
    g = torch.Generator(device="cuda")
    g.manual_seed(5)
    shapes = [("ffn_down.even", 4096, 14336, "Q6_K"), ("ffn_down.odd", 4096, 14336, "Q4_K"),
              ("ffn_gate", 14336, 4096, "Q4_K")]
    jobs, hs, diags = [], {}, {}
    for name, nrow, n, tt in shapes:
        x = torch.randn(nrow, n, device="cuda", generator=g, dtype=torch.float32) * 0.02
        qw = torch.from_numpy(big[n]["diag"].astype(np.float32)).cuda()
        jobs.append(Job(name, tt, "EF", x, qw, f"h{n}"))
        hs[f"h{n}"] = big[n]["H"]
        diags[f"h{n}"] = big[n]["diag"]
    raws, st = Encoder().run(jobs, hs, diags)
    rng = np.random.default_rng(0)
    for j, (name, nrow, n, tt) in zip(jobs, shapes):
        rows = np.sort(np.r_[0, nrow - 1, rng.choice(np.arange(1, nrow - 1), 46, replace=False)])
        W = j.x.cpu().numpy()[rows]
        qw = j.qw.cpu().numpy()
        got = raws[name].cpu().numpy()[rows]
        want, want_recon = orc.ef_encode(W, tt, qw, big[n]["Hh"], n_iter=2, act_order=True, U=oracle_u[n])
        same = float(np.mean(orc.codes(tt, got, *W.shape) == orc.codes(tt, want, *W.shape)))
        e_got = h_weighted_err(W, orc.dequantize(tt, got, n), big[n]["Hh"])
        e_want = h_weighted_err(W, want_recon, big[n]["Hh"])
        print(f"{name} {tt} {nrow}x{n}: codes identical {same:.5%}, bytes identical "
              f"{np.array_equal(got, want)}, H-err ratio {e_got / e_want:.7f}")
        assert same >= 0.999, f"{name}: codes identical {same:.4%}"
        assert abs(e_got / e_want - 1.0) <= 1e-3
    assert all(np.isfinite(v["rel_err_vs_stock"]) for v in st.values())
