"""Host file I/O around the encoder: GGUF containers (pip `gguf`), imatrix means and the
reference's Hessian storage format.

  * copy_gguf(src, dst, replace)   re-emit `src` with the same metadata and tensor list, the
                                   payloads named in `replace` swapped for new k-quant bytes
                                   (the write path of coldpress/ggufio.py:46-85 reemit)
  * imatrix_means(path)            {tensor: in_sum2 / count} (coldpress/ggufio.py:105-123)
  * save_hessians / load_hessian   per-tensor npz with float16 H / hscale, exact float32
                                   diagonal, hscale and n; the old family-keyed layout is
                                   read too (coldpress/hessians.py:185-245)
"""
import os

import numpy as np

FP16_SAFE_MAX = 32768.0
# GGUF tensor name -> family key of the old layout (inputs shared by q/k/v and gate/up)
_FAMILY = {"attn_q": "qkv_in", "attn_k": "qkv_in", "attn_v": "qkv_in", "attn_output": "o_in",
           "ffn_gate": "gateup_in", "ffn_up": "gateup_in", "ffn_down": "down_in"}


# ---------------------------------------------------------------------------- GGUF

def _kv(field):
    """(value, value type, item type) of a reader field, decoded from its parts."""
    from gguf import GGUFValueType
    vt = field.types[0]
    if vt == GGUFValueType.ARRAY:
        it = field.types[1]
        if it == GGUFValueType.STRING:
            return [bytes(field.parts[i]).decode("utf-8") for i in field.data], vt, it
        return [field.parts[i].item() for i in field.data], vt, it
    if vt == GGUFValueType.STRING:
        return bytes(field.parts[field.data[0]]).decode("utf-8"), vt, None
    v = field.parts[field.data[0]].item()
    return (bool(v) if vt == GGUFValueType.BOOL else v), vt, None


def architecture(reader):
    for f in reader.fields.values():
        if f.name == "general.architecture":
            return bytes(f.parts[f.data[0]]).decode("utf-8")
    return None


def copy_gguf(src, dst, replace=None):
    """Write dst as a copy of src (all key/values, all tensors in order) with the raw bytes of
    the quantized tensors in `replace` ({name: uint8 array of the same byte size}) swapped."""
    from gguf import GGUFReader, GGUFWriter
    replace = replace or {}
    r = GGUFReader(src)
    arch = architecture(r)
    if not arch:
        raise ValueError(f"{src}: no general.architecture key")
    w = GGUFWriter(dst, arch)
    internal = {"GGUF.version", "GGUF.tensor_count", "GGUF.kv_count", "general.architecture"}
    for f in r.fields.values():
        if f.name in internal:
            continue
        val, vt, it = _kv(f)
        w.add_key_value(f.name, val, vt, sub_type=it)
    for t in r.tensors:
        data = np.asarray(t.data)
        if t.name in replace:
            new = np.ascontiguousarray(replace[t.name], dtype=np.uint8)
            if data.dtype != np.uint8:
                raise ValueError(f"{t.name}: only quantized payloads can be replaced")
            if new.nbytes != int(t.n_bytes):
                raise ValueError(f"{t.name}: {new.nbytes} bytes for a {int(t.n_bytes)}-byte tensor")
            data = new.reshape(data.shape)
        w.add_tensor(t.name, data, raw_dtype=t.tensor_type)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    return len(replace)


def imatrix_means(path):
    """{tensor name: float32 per-column mean of squared inputs} of an imatrix GGUF."""
    from gguf import GGUFReader
    r = GGUFReader(path)
    sums, counts = {}, {}
    for t in r.tensors:
        if t.name.endswith(".in_sum2"):
            sums[t.name[:-8]] = np.array(t.data, dtype=np.float32)
        elif t.name.endswith(".counts"):
            counts[t.name[:-7]] = np.array(t.data, dtype=np.float32)
    return {k: (s / np.float32(float(counts[k].reshape(-1)[0]))).astype(np.float32) for k, s in sums.items()}


# ---------------------------------------------------------------------------- Hessians

def hessian_file(hessdir, gguf_name):
    return os.path.join(hessdir, gguf_name.replace(".", "_") + ".npz")


def _family_key(gguf_name):
    if gguf_name == "output.weight":
        return "lmhead_in"
    parts = gguf_name.split(".")
    if not gguf_name.startswith("blk.") or len(parts) < 3:
        return None
    fam = _FAMILY.get(parts[2])
    return f"blk.{parts[1]}.{fam}" if fam else None


def hessian_path(hessdir, gguf_name):
    """The npz that holds gguf_name's Hessian (per-tensor file, else the family file)."""
    cands = [hessian_file(hessdir, gguf_name)]
    fk = _family_key(gguf_name)
    if fk is not None:
        cands.append(hessian_file(hessdir, fk))
    for p in cands:
        if os.path.exists(p):
            return p
    raise FileNotFoundError(f"no Hessian for {gguf_name} (tried {cands})")


def has_hessian(hessdir, gguf_name):
    try:
        hessian_path(hessdir, gguf_name)
        return True
    except FileNotFoundError:
        return False


def load_hessian_stored(hessdir, gguf_name):
    """The stored components of a Hessian: dict(h (float16 or float32 [d, d]), diag32 (or None),
    hscale (float), n (int), path).  Decoding to float64 happens on the device
    (cp_hessian_decode) or in load_hessian."""
    path = hessian_path(hessdir, gguf_name)
    z = np.load(path)
    return {"h": np.asarray(z["H"]), "diag32": np.asarray(z["diag32"], np.float32) if "diag32" in z.files else None,
            "hscale": float(z["hscale"]) if "hscale" in z.files else 1.0, "n": int(z["n"]), "path": path}


def load_hessian(hessdir, gguf_name):
    """(H float64 [d, d], n): float64(stored) * hscale with the exact float32 diagonal restored."""
    st = load_hessian_stored(hessdir, gguf_name)
    H = st["h"].astype(np.float64)
    if st["hscale"] != 1.0:
        H *= st["hscale"]
    if st["diag32"] is not None:
        np.fill_diagonal(H, st["diag32"].astype(np.float64))
    return H, st["n"]


def save_hessians(hessians, outdir):
    """{gguf_name: {"H": float32 [d, d], "n": int}} -> one npz per tensor: float16 H / hscale
    (hscale keeps |H| / hscale under FP16_SAFE_MAX), exact float32 diagonal, hscale, n."""
    os.makedirs(outdir, exist_ok=True)
    for name, h in hessians.items():
        H = np.asarray(h["H"], dtype=np.float32)
        amax = float(np.max(np.abs(H))) if H.size else 0.0
        hscale = amax / FP16_SAFE_MAX if amax > FP16_SAFE_MAX else 1.0
        np.savez_compressed(hessian_file(outdir, name), H=(H / np.float32(hscale)).astype(np.float16),
                            diag32=np.ascontiguousarray(np.diag(H)).astype(np.float32), hscale=np.float32(hscale),
                            n=h["n"], name=name)
