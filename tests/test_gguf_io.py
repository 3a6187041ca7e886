"""Host file I/O: GGUF re-emission, imatrix means and the Hessian storage format."""
import numpy as np

import gguf_fixtures as fx


def test_copy_gguf_is_byte_identical_without_replacements(tmp_path, orc):
    from gguf import GGUFReader
    from perm_b200 import gguf_io
    W = fx.weights()
    src, dst = str(tmp_path / "t.gguf"), str(tmp_path / "c.gguf")
    fx.write_target(src, W, orc.quantize)
    gguf_io.copy_gguf(src, dst)
    a, b = GGUFReader(src), GGUFReader(dst)
    assert [t.name for t in a.tensors] == [t.name for t in b.tensors]
    for ta, tb in zip(a.tensors, b.tensors):
        assert ta.tensor_type == tb.tensor_type
        assert np.array_equal(np.asarray(ta.data).view(np.uint8), np.asarray(tb.data).view(np.uint8))
    ka = {f.name: gguf_io._kv(f)[0] for f in a.fields.values() if not f.name.startswith("GGUF.")}
    kb = {f.name: gguf_io._kv(f)[0] for f in b.fields.values() if not f.name.startswith("GGUF.")}
    assert ka == kb


def test_copy_gguf_replaces_payloads_and_checks_size(tmp_path, orc):
    import pytest
    from gguf import GGUFReader
    from perm_b200 import gguf_io
    W = fx.weights()
    src, dst = str(tmp_path / "t.gguf"), str(tmp_path / "c.gguf")
    fx.write_target(src, W, orc.quantize)
    t = {x.name: x for x in GGUFReader(src).tensors}["blk.0.attn_q.weight"]
    new = np.full(int(t.n_bytes), 7, np.uint8)
    gguf_io.copy_gguf(src, dst, {"blk.0.attn_q.weight": new})
    got = {x.name: x for x in GGUFReader(dst).tensors}["blk.0.attn_q.weight"]
    assert np.array_equal(np.asarray(got.data).reshape(-1), new)
    with pytest.raises(ValueError):
        gguf_io.copy_gguf(src, dst, {"blk.0.attn_q.weight": new[:-1]})


def test_hessian_storage_roundtrip(tmp_path):
    from perm_b200 import gguf_io
    hs = fx.hessians()
    gguf_io.save_hessians(hs, str(tmp_path))
    for name, h in hs.items():
        H, n = gguf_io.load_hessian(str(tmp_path), name)
        assert n == h["n"] and H.dtype == np.float64
        assert np.array_equal(np.diag(H), np.diag(h["H"]).astype(np.float64))   # exact diagonal
        off = ~np.eye(H.shape[0], dtype=bool)
        rel = np.abs(H - h["H"])[off] / np.maximum(np.abs(h["H"][off]), 1e-30)
        assert np.all(np.isfinite(H)) and np.median(rel) < 1e-3                # float16 storage
    st = gguf_io.load_hessian_stored(str(tmp_path), "blk.0.attn_q.weight")
    assert st["hscale"] > 1.0 and st["h"].dtype == np.float16                  # overflow guard active


def test_family_layout_fallback(tmp_path):
    from perm_b200 import gguf_io
    H = np.eye(256, dtype=np.float32) * 3
    np.savez(str(tmp_path / "blk_2_qkv_in.npz"), H=H, n=10)
    Hk, n = gguf_io.load_hessian(str(tmp_path), "blk.2.attn_k.weight")
    assert n == 10 and np.array_equal(Hk, H.astype(np.float64))
    assert gguf_io.has_hessian(str(tmp_path), "blk.2.attn_v.weight")
    assert not gguf_io.has_hessian(str(tmp_path), "blk.2.ffn_up.weight")


def test_imatrix_means(tmp_path):
    from perm_b200 import gguf_io
    p = str(tmp_path / "im.gguf")
    fx.write_imatrix(p, [("blk.0.attn_q.weight", 256)])
    m = gguf_io.imatrix_means(p)
    assert m["blk.0.attn_q.weight"].shape == (256,) and m["blk.0.attn_q.weight"].dtype == np.float32


def test_encode_gguf_rejects_unsupported_types_before_touching_a_gpu(tmp_path):
    import gguf
    import pytest
    from gguf import GGUFWriter
    from perm_b200 import ef
    p = str(tmp_path / "bad.gguf")
    w = GGUFWriter(p, "qwen3")
    w.add_tensor("x.weight", np.zeros((4, 36), np.uint8), raw_shape=(4, 36),
                 raw_dtype=gguf.GGMLQuantizationType.Q4_0)
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()
    with pytest.raises(ValueError, match="cannot encode"):
        ef.encode_gguf(p, p, str(tmp_path), str(tmp_path / "o.gguf"), log=lambda *_: None)
