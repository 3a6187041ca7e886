"""Tensor inventories of the whole-model encode workloads and their synthetic inputs.

A model is described by its GGUF tensor names and shapes ([out, in] row-major, the layout
ef.py reads from a GGUF), the k-quant type of each tensor and the Hessian that feeds its error
feedback.  q/k/v share one input (and so one Hessian), gate/up share another; the GGUF
Hessian files the reference's collector writes for them hold identical matrices
(coldpress/hessians.py:137-152), so the encoder factorises each distinct input once.

Type maps:
  * "q2_k_mix" (Qwen3-0.6B recipe, paper/METHOD.md:72-73): Q2_K for attn_q, attn_k,
    ffn_gate, ffn_up and token_embd; Q3_K for attn_v, attn_output, ffn_down; Q6_K output.
  * "q4_k_m_style": Q4_K everywhere; Q6_K for output and for attn_v / ffn_down of even
    layers.  llama.cpp's own Q4_K_M layer rule is not part of the reference, so this fixed,
    deterministic rule stands in for it.
"""
from dataclasses import dataclass

import numpy as np

QWEN3_06B = dict(name="qwen3-0.6b", n_layers=28, hidden=1024, n_q=16, n_kv=8, head_dim=128, ffn=3072,
                 vocab=151936)
LLAMA3_8B = dict(name="llama3-8b", n_layers=32, hidden=4096, n_q=32, n_kv=8, head_dim=128, ffn=14336,
                 vocab=128256)
MODELS = {"qwen3-0.6b": QWEN3_06B, "llama3-8b": LLAMA3_8B}


@dataclass
class TensorSpec:
    name: str
    nrow: int
    n: int
    ttype: str
    mode: str            # "EF", "wRTN" or "wRTN(attn0-diag)" (ef.py:278-297)
    hkey: str = None     # Hessian feeding EF (and the imatrix means)

    @property
    def params(self):
        return self.nrow * self.n


def _type_for(kind, layer, mixture):
    if mixture == "q2_k_mix":
        return {"attn_q": "Q2_K", "attn_k": "Q2_K", "ffn_gate": "Q2_K", "ffn_up": "Q2_K",
                "attn_v": "Q3_K", "attn_output": "Q3_K", "ffn_down": "Q3_K",
                "token_embd": "Q2_K", "output": "Q6_K"}[kind]
    if mixture == "q4_k_m_style":
        if kind == "output":
            return "Q6_K"
        if kind in ("attn_v", "ffn_down") and layer % 2 == 0:
            return "Q6_K"
        return "Q4_K"
    raise ValueError(mixture)


def tensor_specs(cfg, mixture):
    """GGUF tensors of the model in the reference's encode order (blocks, then embd/output)."""
    h, hd = cfg["hidden"], cfg["head_dim"]
    q_out, kv_out, ffn = cfg["n_q"] * hd, cfg["n_kv"] * hd, cfg["ffn"]
    specs = []
    for i in range(cfg["n_layers"]):
        b = f"blk.{i}."
        shapes = [("attn_q", q_out, h, "qkv"), ("attn_k", kv_out, h, "qkv"), ("attn_v", kv_out, h, "qkv"),
                  ("attn_output", h, q_out, "o"), ("ffn_gate", ffn, h, "gateup"), ("ffn_up", ffn, h, "gateup"),
                  ("ffn_down", h, ffn, "down")]
        for kind, nrow, n, hk in shapes:
            specs.append(TensorSpec(b + kind + ".weight", nrow, n, _type_for(kind, i, mixture), "EF", f"blk.{i}.{hk}"))
    specs.append(TensorSpec("token_embd.weight", cfg["vocab"], h, _type_for("token_embd", 0, mixture),
                            "wRTN(attn0-diag)", "blk.0.qkv"))
    specs.append(TensorSpec("output.weight", cfg["vocab"], h, _type_for("output", 0, mixture), "EF", "output"))
    return specs


def hessian_dims(specs):
    """{hkey: d} of every distinct Hessian the specs use."""
    out = {}
    for s in specs:
        if s.hkey is not None:
            out[s.hkey] = s.n
    return out


def synth_weights(torch, spec, seed, device):
    """Random-init weights N(0, 0.02), float32 [nrow, n], reproducible per (seed, tensor)."""
    g = torch.Generator(device=device)
    g.manual_seed((seed * 1000003 + _stable_hash(spec.name)) % (2 ** 63))
    return torch.randn((spec.nrow, spec.n), generator=g, device=device, dtype=torch.float32).mul_(0.02)


def synth_hessian(torch, d, key, seed, device, tokens=262144, chunk=32768):
    """H = X^T X / T for X = N(0, 1) * per-channel log-normal(0, 1) scales, T tokens of bf16
    activations (the Hessian-collection workload, accumulated by this library's X^T X
    kernel); returned float64 [d, d]."""
    from . import hessians
    g = torch.Generator(device=device)
    g.manual_seed((seed * 7919 + _stable_hash(key)) % (2 ** 63))
    scales = torch.exp(torch.randn(d, generator=g, device=device, dtype=torch.float32))
    H = torch.zeros((d, d), device=device, dtype=torch.float32)
    done = 0
    while done < tokens:
        t = min(chunk, tokens - done)
        X = (torch.randn((t, d), generator=g, device=device, dtype=torch.float32) * scales).to(torch.bfloat16)
        hessians.xtx_accumulate(X, H)
        done += t
    return H.double() / tokens


def _stable_hash(s):
    h = 1469598103934665603
    for ch in s.encode():
        h = ((h ^ ch) * 1099511628211) % (2 ** 64)
    return h % (2 ** 31)


def summary(specs):
    n_params = sum(s.params for s in specs)
    by_type = {}
    for s in specs:
        by_type[s.ttype] = by_type.get(s.ttype, 0) + 1
    return {"tensors": len(specs), "params": n_params, "types": by_type}


if __name__ == "__main__":
    for m in MODELS:
        for mix in ("q2_k_mix", "q4_k_m_style"):
            sp = tensor_specs(MODELS[m], mix)
            print(m, mix, summary(sp), np.unique([s.n for s in sp]))
