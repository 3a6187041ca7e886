"""Synthetic GGUF artefacts for the encode_gguf tests (no downloads, seconds to build)."""
import numpy as np

# (name, target type, ne0 = n_per_row, nrow)
SPEC = [
    ("token_embd.weight", "Q2_K", 256, 384),
    ("output.weight", "Q6_K", 256, 320),
    ("blk.0.attn_q.weight", "Q2_K", 256, 256),
    ("blk.0.attn_k.weight", "Q3_K", 256, 128),
    ("blk.0.attn_v.weight", "Q4_K", 256, 128),
    ("blk.0.ffn_down.weight", "Q5_K", 512, 256),
    ("blk.0.ffn_up.weight", "Q4_K", 256, 512),      # no Hessian: plain weighted RTN
]


def weights():
    rng = np.random.default_rng(11)
    return {name: ((rng.standard_normal((nrow, ne0)) ** 3) * 0.05).astype(np.float32)
            for name, tt, ne0, nrow in SPEC}


def write_f16(path, W):
    from gguf import GGUFWriter
    w = GGUFWriter(path, "qwen3")
    w.add_uint32("qwen3.block_count", 1)
    w.add_string("general.name", "synthetic")
    for name, arr in W.items():
        w.add_tensor(name, arr.astype(np.float16))
    w.add_tensor("blk.0.attn_norm.weight", np.ones(256, np.float32))
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()


def write_target(path, W, quantize):
    import gguf
    from gguf import GGUFWriter
    w = GGUFWriter(path, "qwen3")
    w.add_uint32("qwen3.block_count", 1)
    w.add_string("general.name", "synthetic")
    for name, tt, ne0, nrow in SPEC:
        raw = quantize(tt, W[name].astype(np.float16).astype(np.float32), None)
        w.add_tensor(name, np.ascontiguousarray(raw, np.uint8), raw_shape=raw.shape,
                     raw_dtype=getattr(gguf.GGMLQuantizationType, tt))
    w.add_tensor("blk.0.attn_norm.weight", np.ones(256, np.float32))
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()


def write_imatrix(path, names_ne0):
    from gguf import GGUFWriter
    rng = np.random.default_rng(5)
    w = GGUFWriter(path, "imatrix")
    for name, ne0 in names_ne0:
        w.add_tensor(name + ".in_sum2", (rng.lognormal(0, 1, ne0) * 100).astype(np.float32))
        w.add_tensor(name + ".counts", np.array([100.0], np.float32))
    w.write_header_to_file(); w.write_kv_data_to_file(); w.write_tensors_to_file(); w.close()


def hessians(big=False):
    """Per-tensor Hessians (float32, token counts) for every tensor but token_embd and ffn_up;
    attn_q's has entries above the float16 range, exercising hscale."""
    rng = np.random.default_rng(21)
    out = {}
    for name, tt, ne0, nrow in SPEC:
        if name in ("token_embd.weight", "blk.0.ffn_up.weight"):
            continue
        X = rng.standard_normal((2048, ne0)) * rng.lognormal(0, 1, ne0)
        X += 0.3 * X[:, [0]]
        H = (X.T @ X).astype(np.float32)
        if name == "blk.0.attn_q.weight":
            H *= 50.0
        out[name] = {"H": H, "n": 2048}
    return out
