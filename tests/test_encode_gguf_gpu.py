"""encode_gguf(device="cuda") end to end on a synthetic model: every output tensor must match
the reference semantics (EF with its Hessian, attn0-diagonal weighted RTN for token_embd,
weighted RTN without a Hessian), computed by the CPU oracle from the same files."""
import json

import numpy as np
import pytest

import gguf_fixtures as fx

pytestmark = pytest.mark.gpu


def test_encode_gguf_matches_reference_semantics(tmp_path, orc):
    from gguf import GGUFReader
    from perm_b200 import ef, gguf_io
    W = fx.weights()
    f16, tgt, out = str(tmp_path / "f16.gguf"), str(tmp_path / "t.gguf"), str(tmp_path / "o.gguf")
    hdir, imp = str(tmp_path / "hess"), str(tmp_path / "im.gguf")
    fx.write_f16(f16, W)
    fx.write_target(tgt, W, orc.quantize)
    gguf_io.save_hessians(fx.hessians(), hdir)
    fx.write_imatrix(imp, [(n, ne0) for n, tt, ne0, nrow in fx.SPEC if n != "token_embd.weight"])
    stats = ef.encode_gguf(f16, tgt, hdir, out, imatrix_path=imp, log=lambda *_: None)
    imat = gguf_io.imatrix_means(imp)
    got = {t.name: np.asarray(t.data) for t in GGUFReader(out).tensors}
    for name, tt, ne0, nrow in fx.SPEC:
        x = W[name].astype(np.float16).astype(np.float32)
        qw = imat.get(name)
        if name == "token_embd.weight":
            H0, n0 = gguf_io.load_hessian(hdir, "blk.0.attn_q.weight")
            want = orc.quantize(tt, x, (np.diag(H0) / n0).astype(np.float32))
            assert stats[name]["mode"] == "wRTN(attn0-diag)"
            assert np.array_equal(got[name].reshape(want.shape), want)
        elif gguf_io.has_hessian(hdir, name):
            H, _ = gguf_io.load_hessian(hdir, name)
            want, _ = orc.ef_encode(x, tt, qw, H, n_iter=2, act_order=True)
            g = got[name].reshape(want.shape)
            frac = float(np.mean(orc.codes(tt, g, nrow, ne0) == orc.codes(tt, want, nrow, ne0)))
            assert stats[name]["mode"] == "EF"
            assert frac >= 0.999, f"{name}: codes identical {frac:.4%}"
        else:
            want = orc.quantize(tt, x, qw)
            assert stats[name]["mode"] == "wRTN"
            assert np.array_equal(got[name].reshape(want.shape), want)
    assert np.array_equal(got["blk.0.attn_norm.weight"], np.ones(256, np.float32))
    on_disk = json.load(open(out + ".efstats.json"))
    assert set(on_disk) == {n for n, *_ in fx.SPEC}
    assert all(np.isfinite(v["rel_err_vs_stock"]) for v in on_disk.values())




def test_encode_gguf_batches_and_timings(tmp_path, orc):
    """Small batches (several in flight through Encoder.run_stream, each tensor's inputs
    uploaded in storage form and decoded on the device) give exactly the bytes and statistics
    of one batch, and the timings record is filled."""
    from gguf import GGUFReader
    from perm_b200 import ef, gguf_io
    W = fx.weights()
    f16, tgt = str(tmp_path / "f16.gguf"), str(tmp_path / "t.gguf")
    hdir, imp = str(tmp_path / "hess"), str(tmp_path / "im.gguf")
    fx.write_f16(f16, W)
    fx.write_target(tgt, W, orc.quantize)
    gguf_io.save_hessians(fx.hessians(), hdir)
    fx.write_imatrix(imp, [(n, ne0) for n, tt, ne0, nrow in fx.SPEC if n != "token_embd.weight"])
    one, many = str(tmp_path / "one.gguf"), str(tmp_path / "many.gguf")
    st1 = ef.encode_gguf(f16, tgt, hdir, one, imatrix_path=imp, log=lambda *_: None)
    tm = {}
    st2 = ef.encode_gguf(f16, tgt, hdir, many, imatrix_path=imp, log=lambda *_: None, max_params_per_batch=100_000,
                         timings=tm)
    a = {t.name: np.asarray(t.data) for t in GGUFReader(one).tensors}
    b = {t.name: np.asarray(t.data) for t in GGUFReader(many).tensors}
    assert a.keys() == b.keys()
    for k in a:
        assert np.array_equal(a[k], b[k]), k
    assert list(st1) == list(st2) == [n for n, *_ in fx.SPEC]
    for k in st1:
        assert st1[k]["rel_err_vs_stock"] == pytest.approx(st2[k]["rel_err_vs_stock"], rel=1e-9, abs=1e-12)
        assert set(st1[k]) == {"type", "mode", "rel_err_vs_stock", "sec"}
    assert tm["batches"] >= 4 and tm["tensors"] == len(fx.SPEC)
    assert tm["h2d_bytes"] > 0 and tm["d2h_bytes"] > 0 and tm["wall_s"] >= tm["write_s"]


class _PermSpacemap:
    """Stand-in for a PERM spacemap (perm/spacemaps): input_perm(name, perms, dims) returns the
    input permutation of a tensor, or None for tensors it does not permute."""

    def __init__(self, table):
        self.table = table

    def input_perm(self, name, perms, dims, **_):
        return self.table.get(name)


def test_encode_gguf_with_input_permutations(tmp_path, orc):
    """ef.py:289-290 and 272-276: with PERM permutations the imatrix and the Hessian are
    permuted (qw[p], H[p][:, p]) while the weights are read as stored; token_embd's fit
    weights are permuted too.  Every output must match the oracle run on the permuted inputs,
    and identical Hessians under different permutations must not be shared."""
    from gguf import GGUFReader
    from perm_b200 import ef, gguf_io
    W = fx.weights()
    f16, tgt, out = str(tmp_path / "f16.gguf"), str(tmp_path / "t.gguf"), str(tmp_path / "o.gguf")
    hdir, imp = str(tmp_path / "hess"), str(tmp_path / "im.gguf")
    fx.write_f16(f16, W)
    fx.write_target(tgt, W, orc.quantize)
    gguf_io.save_hessians(fx.hessians(), hdir)
    fx.write_imatrix(imp, [(n, ne0) for n, tt, ne0, nrow in fx.SPEC if n != "token_embd.weight"])
    rng = np.random.default_rng(17)
    ne0 = {n: e for n, tt, e, nrow in fx.SPEC}
    table = {n: rng.permutation(ne0[n]) for n in ("token_embd.weight", "blk.0.attn_q.weight",
                                                  "blk.0.ffn_down.weight", "blk.0.ffn_up.weight")}
    stats = ef.encode_gguf(f16, tgt, hdir, out, imatrix_path=imp, perms={"any": 1}, spacemap=_PermSpacemap(table),
                           log=lambda *_: None, max_params_per_batch=150_000)
    imat = gguf_io.imatrix_means(imp)
    got = {t.name: np.asarray(t.data) for t in GGUFReader(out).tensors}
    for name, tt, e, nrow in fx.SPEC:
        x = W[name].astype(np.float16).astype(np.float32)
        p = table.get(name)
        qw = imat.get(name)
        if qw is not None and p is not None:
            qw = qw[p]
        if name == "token_embd.weight":
            H0, n0 = gguf_io.load_hessian(hdir, "blk.0.attn_q.weight")
            fw = (np.diag(H0) / n0).astype(np.float32)
            want = orc.quantize(tt, x, fw[p] if p is not None else fw)
            assert np.array_equal(got[name].reshape(want.shape), want), name
        elif gguf_io.has_hessian(hdir, name):
            H, _ = gguf_io.load_hessian(hdir, name)
            if p is not None:
                H = H[np.ix_(p, p)]
            want, _ = orc.ef_encode(x, tt, qw, H, n_iter=2, act_order=True)
            g = got[name].reshape(want.shape)
            frac = float(np.mean(orc.codes(tt, g, nrow, e) == orc.codes(tt, want, nrow, e)))
            assert frac >= 0.999, f"{name}: codes identical {frac:.4%}"
        else:
            want = orc.quantize(tt, x, qw)
            assert np.array_equal(got[name].reshape(want.shape), want), name
    assert set(stats) == {n for n, *_ in fx.SPEC}
