"""Memory-bounded streaming (Encoder.run_stream over perm_b200.stream batches): a model cut
into several batches, each decoding its own storage-form Hessians, must give exactly the
bytes and statistics of one Encoder.run over all tensors with the same decoded Hessians, and
a non-positive-definite Hessian inside a batch must still take the reference's damp
escalation (ef.py:67-76) and match the oracle."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _setup(torch, seed, layers=5, bad_layer=None):
    from perm_b200 import stream as stm
    from perm_b200.encoder import Job
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    stored, dims, jobs = {}, {}, []
    for L in range(layers):
        for hk, n in ((f"l{L}.a", 512), (f"l{L}.b", 1024)):
            X = torch.randn(2048, n, device="cuda", dtype=torch.float64, generator=g)
            X *= torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
            H = X.T @ X / 2048
            if bad_layer == L and hk.endswith(".a"):   # one clearly negative eigenvalue
                Q, _ = torch.linalg.qr(torch.randn(n, n, device="cuda", dtype=torch.float64, generator=g))
                eig = torch.linspace(1.0, 100.0, n, device="cuda", dtype=torch.float64)
                eig[0] = -2.0
                H = (Q * eig) @ Q.T
                H = (H + H.T) / 2
            stored[hk] = stm.store_hessian(torch, H)
            dims[hk] = n
        for i, (hk, rows, tt) in enumerate(((f"l{L}.a", 300, "Q2_K"), (f"l{L}.a", 200, "Q3_K"),
                                            (f"l{L}.b", 256, "Q4_K"), (f"l{L}.b", 128, "Q6_K"))):
            n = dims[hk]
            x = torch.randn(rows, n, device="cuda", generator=g, dtype=torch.float32) * 0.02
            qw = torch.from_numpy(np.abs(stored[hk].diag_host).astype(np.float32)).cuda()
            jobs.append(Job(f"l{L}.t{i}", tt, "EF", x, qw, hk))
    emb = torch.randn(333, 512, device="cuda", generator=g, dtype=torch.float32) * 0.02
    fw = torch.from_numpy(stored["l0.a"].diag_host.astype(np.float32)).cuda()
    jobs.append(Job("embd", "Q2_K", "wRTN(attn0-diag)", emb, fw, None, fit_w=fw))
    jobs.append(Job("plain", "Q5_K", "wRTN", torch.randn(64, 512, device="cuda", generator=g) * 0.02, None, None))
    return stored, dims, jobs


def test_stream_matches_one_pass():
    import torch
    from perm_b200 import stream as stm
    from perm_b200.encoder import Encoder
    stored, dims, jobs = _setup(torch, 7)
    s = torch.cuda.current_stream()
    hd = {k: stm.decode(torch, v, s) for k, v in stored.items()}
    diags = {k: v.diag_host for k, v in stored.items()}
    want, st_want = Encoder().run(jobs, hd, diags)
    budget = 2 * stm.hessian_bytes(1024) + 2 * stm.hessian_bytes(512) + 200_000 * stm.ef_bytes_per_param()
    plan = stm.plan(jobs, dims, budget)
    assert len(plan) >= 3
    assert sorted(j.name for b in plan for j in b) == sorted(j.name for j in jobs)
    for b in plan:   # a Hessian's jobs never straddle two batches
        for other in plan:
            if other is not b:
                assert not ({j.hkey for j in b if j.mode == "EF"} & {j.hkey for j in other if j.mode == "EF"})
    seen = []
    got, st_got = Encoder().run_stream(stm.batches(torch, plan, stored),
                                       on_batch=lambda b, r, st: seen.append(sorted(r)))
    assert len(seen) == len(plan)
    for j in jobs:
        a, b = got[j.name].cpu().numpy(), want[j.name].cpu().numpy()
        assert np.array_equal(a, b), f"{j.name}: {np.count_nonzero(a != b)} bytes differ"
        # the statistics' float64 sums are reduced with atomics: equal up to summation order
        assert st_got[j.name]["rel_err_vs_stock"] == pytest.approx(st_want[j.name]["rel_err_vs_stock"],
                                                                   rel=1e-9, abs=1e-12)


def test_stream_escalates_inside_a_batch(orc):
    import torch
    from perm_b200 import stream as stm
    from perm_b200.encoder import Encoder
    stored, dims, jobs = _setup(torch, 8, layers=3, bad_layer=1)
    budget = stm.hessian_bytes(1024) + stm.hessian_bytes(512) + 300_000 * stm.ef_bytes_per_param()
    plan = stm.plan(jobs, dims, budget)
    assert len(plan) >= 3
    got, _ = Encoder().run_stream(stm.batches(torch, plan, stored))
    s = torch.cuda.current_stream()
    for j in jobs:
        if j.hkey != "l1.a":
            continue
        H = stm.decode(torch, stored[j.hkey], s).cpu().numpy()
        W = j.x.cpu().numpy()
        want, _ = orc.ef_encode(W, j.ttype, j.qw.cpu().numpy(), H, n_iter=2, act_order=True)
        g = got[j.name].cpu().numpy()
        frac = float(np.mean(orc.codes(j.ttype, g, *W.shape) == orc.codes(j.ttype, want, *W.shape)))
        assert frac >= 0.999, f"{j.name}: codes identical {frac:.4%}"
