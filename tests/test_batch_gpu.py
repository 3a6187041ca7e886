"""Grouped (multi-tensor) launches vs the oracle: the whole-model encoder must produce the
same bytes as the per-tensor reference semantics."""
import numpy as np
import pytest

from conftest import K_TYPES

pytestmark = pytest.mark.gpu


def _hessian(rng, n, T=2048):
    X = rng.standard_normal((T, n)) * rng.lognormal(0, 1, n)
    return X.T @ X / T


def _encode(jobs_np, hess_np, stats=True):
    import torch
    from perm_b200.encoder import Encoder, Job
    hd = {k: torch.from_numpy(H).cuda() for k, H in hess_np.items()}
    diags = {k: np.diag(H) for k, H in hess_np.items()}
    jobs = []
    for name, tt, mode, W, qw, hk, fw in jobs_np:
        jobs.append(Job(name, tt, mode, torch.from_numpy(W).cuda(),
                        None if qw is None else torch.from_numpy(qw).cuda(), hk,
                        None if fw is None else torch.from_numpy(fw).cuda()))
    enc = Encoder()
    factors = enc.factor(hd, diags)
    raws, st = enc.encode(jobs, factors, stats=stats)
    return {k: v.cpu().numpy() for k, v in raws.items()}, st


@pytest.mark.parametrize("many_rows", [False, True])
def test_grouped_encode_matches_oracle(orc, many_rows):
    rng = np.random.default_rng(3)
    n = 256
    hess = {"a": _hessian(rng, n), "b": _hessian(rng, 512)}
    rows = 1024 if many_rows else 40      # 20 x 1024 rows: several CTAs per tensor
    jobs = []
    for i in range(20 if many_rows else 6):
        tt = K_TYPES[i % 5]
        hk = "a" if i % 2 == 0 else "b"
        nn = hess[hk].shape[0]
        W = (rng.standard_normal((rows if i else rows + 3, nn)) * 0.02).astype(np.float32)
        jobs.append((f"t{i}", tt, "EF", W, np.diag(hess[hk]).astype(np.float32), hk, None))
    Wemb = (rng.standard_normal((77, n)) * 0.02).astype(np.float32)
    jobs.append(("embd", "Q2_K", "wRTN(attn0-diag)", Wemb, None, "a", np.diag(hess["a"]).astype(np.float32)))
    got, st = _encode(jobs, hess)
    for name, tt, mode, W, qw, hk, fw in jobs:
        if mode == "EF":
            want, _ = orc.ef_encode(W, tt, qw, hess[hk], n_iter=2, act_order=True)
        else:
            want = orc.quantize(tt, W, fw)
        assert np.array_equal(got[name], want), f"{name} {tt}: {np.count_nonzero(got[name] != want)} bytes differ"
    assert set(st) == {j[0] for j in jobs}
    assert all(np.isfinite(v["rel_err_vs_stock"]) for v in st.values())


def test_grouped_stats_match_reference_formula(orc):
    rng = np.random.default_rng(9)
    H = _hessian(rng, 512)
    W = (rng.standard_normal((64, 512)) * 0.02).astype(np.float32)
    qw = np.diag(H).astype(np.float32)
    got, st = _encode([("w", "Q3_K", "EF", W, qw, "h", None)], {"h": H})
    recon = orc.dequantize("Q3_K", got["w"], 512)
    base = orc.roundtrip(W, "Q3_K", qw)
    e_ours = float(((((recon - W) ** 2) * qw).astype(np.float64)).sum())
    e_base = float(((((base - W) ** 2) * qw).astype(np.float64)).sum())
    assert abs(st["w"]["rel_err_vs_stock"] - (e_ours / e_base - 1)) < 1e-6


def test_run_escalates_damp_for_an_indefinite_hessian(orc):
    """Encoder.run overlaps the factorisations with the first fits and reads the status words
    at the end; a Hessian with a clearly negative eigenvalue must be re-factorised with the
    reference's escalated damping and its tensor re-encoded, matching the oracle."""
    import torch
    from perm_b200.encoder import Encoder, Job
    rng = np.random.default_rng(4)
    n = 256
    Q, _ = np.linalg.qr(rng.standard_normal((n, n)))
    eig = np.linspace(1.0, 100.0, n)
    eig[0] = -2.0
    Hbad = (Q * eig) @ Q.T
    Hbad = (Hbad + Hbad.T) / 2
    Hgood = _hessian(rng, n)
    W1 = (rng.standard_normal((64, n)) * 0.02).astype(np.float32)
    W2 = (rng.standard_normal((48, n)) * 0.02).astype(np.float32)
    q1 = np.abs(np.diag(Hbad)).astype(np.float32)
    q2 = np.diag(Hgood).astype(np.float32)
    jobs = [Job("bad", "Q4_K", "EF", torch.from_numpy(W1).cuda(), torch.from_numpy(q1).cuda(), "bad"),
            Job("good", "Q2_K", "EF", torch.from_numpy(W2).cuda(), torch.from_numpy(q2).cuda(), "good")]
    hs = {"bad": torch.from_numpy(Hbad).cuda(), "good": torch.from_numpy(Hgood).cuda()}
    raws, st = Encoder().run(jobs, hs, {"bad": np.diag(Hbad), "good": np.diag(Hgood)})
    for name, tt, W, qw, H in (("bad", "Q4_K", W1, q1, Hbad), ("good", "Q2_K", W2, q2, Hgood)):
        want, _ = orc.ef_encode(W, tt, qw, H, n_iter=2, act_order=True)
        got = raws[name].cpu().numpy()
        frac = float(np.mean(orc.codes(tt, got, *W.shape) == orc.codes(tt, want, *W.shape)))
        assert frac >= 0.999, f"{name}: codes identical {frac:.4%}"


def test_run_with_staged_weights_matches_resident():
    """Encoder.run with the weights arriving in groups on another stream (a list of (event,
    job names), each group's first fits waiting only for its own event) gives the same bytes
    as a run whose weights were on the device from the start."""
    import torch
    from perm_b200.encoder import Encoder, Job
    rng = np.random.default_rng(21)
    hess = {"a": _hessian(rng, 256), "b": _hessian(rng, 512)}
    hd = {k: torch.from_numpy(H).cuda() for k, H in hess.items()}
    diags = {k: np.diag(H) for k, H in hess.items()}
    specs = []
    for i in range(6):
        hk = "a" if i % 2 == 0 else "b"
        W = (rng.standard_normal((96 + 32 * i, hess[hk].shape[0])) * 0.02).astype(np.float32)
        specs.append((f"t{i}", ["Q2_K", "Q3_K", "Q6_K"][i % 3], W, np.diag(hess[hk]).astype(np.float32), hk))
    Wemb = (rng.standard_normal((77, 256)) * 0.02).astype(np.float32)
    fw = torch.from_numpy(np.diag(hess["a"]).astype(np.float32)).cuda()

    def jobs_for(dev_w):
        js = [Job(nm, tt, "EF", dev_w[nm], torch.from_numpy(qw).cuda(), hk) for nm, tt, _, qw, hk in specs]
        js.append(Job("embd", "Q2_K", "wRTN(attn0-diag)", dev_w["embd"], None, None, fit_w=fw))
        return js

    host = {nm: torch.from_numpy(W).pin_memory() for nm, _, W, _, _ in specs}
    host["embd"] = torch.from_numpy(Wemb).pin_memory()
    resident = {nm: h.cuda() for nm, h in host.items()}
    want, st_want = Encoder().run(jobs_for(resident), hd, diags)
    want = {k: v.cpu().numpy() for k, v in want.items()}

    staged_w = {nm: torch.empty_like(resident[nm]) for nm in host}
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    groups = [["t3", "embd"], ["t0", "t1", "t2"], ["t4", "t5"]]
    staged = []
    with torch.cuda.stream(side):
        for g in groups:
            for nm in g:
                staged_w[nm].copy_(host[nm], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(side)
            staged.append((ev, g))
    got, st_got = Encoder().run(jobs_for(staged_w), hd, diags, inputs_event=staged)
    for nm in want:
        assert np.array_equal(got[nm].cpu().numpy(), want[nm]), nm
    assert set(st_got) == set(st_want)
    for k in st_want:   # float64 sums reduced on the device in no fixed order
        assert st_got[k]["rel_err_vs_stock"] == pytest.approx(st_want[k]["rel_err_vs_stock"], rel=1e-9, abs=1e-12)


def test_small_launch_long_rows_match_oracle(orc):
    """A grouped launch too small to fill the GPU sends the rows of long tensors (n >= 2048)
    to the column-split sweep (two warps per 32 rows); the bytes must still be the
    reference's, ragged row counts included."""
    rng = np.random.default_rng(17)
    n = 2048
    hess = {"a": _hessian(rng, n, T=4096)}
    qw = np.diag(hess["a"]).astype(np.float32)
    jobs = []
    for i, (tt, rows) in enumerate((("Q2_K", 96), ("Q3_K", 33), ("Q6_K", 64), ("Q4_K", 1))):
        W = (rng.standard_normal((rows, n)) * 0.02).astype(np.float32)
        jobs.append((f"t{i}", tt, "EF", W, qw, "a", None))
    got, _ = _encode(jobs, hess)
    for name, tt, mode, W, qw_, hk, fw in jobs:
        want, _ = orc.ef_encode(W, tt, qw_, hess[hk], n_iter=2, act_order=True)
        assert np.array_equal(got[name], want), f"{name} {tt}: {np.count_nonzero(got[name] != want)} bytes differ"


def test_medium_launch_matches_oracle(orc):
    """A grouped launch of one and a half to two waves of ordinary sweep CTAs runs the
    two-warp column split (smaller launches take the four-warp one); the bytes must be the
    reference's."""
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    rng = np.random.default_rng(23)
    hess = {"a": _hessian(rng, 256), "b": _hessian(rng, 512)}
    rows = 7 * sms * 128 - 77            # about 7 * sms ordinary 128-row CTAs: 1.75 waves of 4 per SM
    jobs = [("big", "Q2_K", "EF", (rng.standard_normal((rows, 256)) * 0.02).astype(np.float32),
             np.diag(hess["a"]).astype(np.float32), "a", None),
            ("small", "Q3_K", "EF", (rng.standard_normal((45, 512)) * 0.02).astype(np.float32),
             np.diag(hess["b"]).astype(np.float32), "b", None)]
    got, _ = _encode(jobs, hess, stats=False)
    for name, tt, mode, W, qw, hk, fw in jobs:
        want, _ = orc.ef_encode(W, tt, qw, hess[hk], n_iter=2, act_order=True)
        assert np.array_equal(got[name], want), f"{name} {tt}: {np.count_nonzero(got[name] != want)} bytes differ"


def test_nvtx_ranges_change_nothing():
    """Encoder(nvtx=True) wraps every stage's launches in NVTX ranges (for nsys / ncu --nvtx):
    the bytes and statistics are those of the unannotated run."""
    import torch
    from perm_b200.encoder import Encoder, Job
    rng = np.random.default_rng(12)
    H = _hessian(rng, 512)
    hd = {"h": torch.from_numpy(H).cuda()}
    W = (rng.standard_normal((200, 512)) * 0.02).astype(np.float32)
    jobs = [Job("t", "Q4_K", "EF", torch.from_numpy(W).cuda(), torch.from_numpy(np.diag(H).astype(np.float32)).cuda(),
                "h")]
    a, sa = Encoder(nvtx=False).run(jobs, hd, {"h": np.diag(H)})
    b, sb = Encoder(nvtx=True).run(jobs, hd, {"h": np.diag(H)})
    assert np.array_equal(a["t"].cpu().numpy(), b["t"].cpu().numpy())
    assert sa["t"]["rel_err_vs_stock"] == pytest.approx(sb["t"]["rel_err_vs_stock"], rel=1e-9)
