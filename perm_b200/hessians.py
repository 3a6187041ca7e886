"""Hessian collection on the GPU (coldpress/hessians.py:402-496).

The reference hook computes `x.float(); acc += (x.T @ x).to(cpu)` for every hooked matmul.
Here the accumulator stays on the device in float32 and each batch's X^T X is accumulated by
the library's tensor-core kernel straight from the bf16 activations (bf16 products are exact
in float32, so only the summation order differs from the reference's float32 matmul).
collect_hessians keeps the reference's name mapping, shape cross-check and return format.
"""
import numpy as np

from . import _native as nat


def xtx_accumulate(x, H, stream=None):
    """H += x^T x.  x: torch bf16 CUDA [T, d] (contiguous), H: torch f32 CUDA [d, d]."""
    torch = nat.torch_cuda()
    if x.dtype != torch.bfloat16:
        raise ValueError("xtx_accumulate expects bf16 activations")
    T, d = x.shape
    if H.shape != (d, d) or H.dtype != torch.float32:
        raise ValueError(f"H must be float32 [{d}, {d}]")
    nat.check(nat.lib().cp_xtx_accumulate(nat.ptr(x), T, d, nat.ptr(H), nat.stream_ptr(torch, stream)),
              "xtx_accumulate")
    return H


def _block_index(gguf_name):
    """Block index of a GGUF tensor name, or -1 for embd/output/norm (hessians.py:53-60)."""
    if gguf_name.startswith("blk."):
        try:
            return int(gguf_name.split(".")[1])
        except (IndexError, ValueError):
            return -1
    return -1


def build_name_map(model, arch, n_layers):
    """{module_name: gguf_base_name} through gguf's TensorNameMap, as hessians.py:63-82."""
    import gguf
    import torch.nn as nn
    inv = {v: k for k, v in gguf.MODEL_ARCH_NAMES.items()}
    enum = inv.get(arch)
    if enum is None:
        raise ValueError(f"arch {arch!r} is unknown to the installed gguf package; "
                         f"cannot map module names to GGUF tensor names")
    nm = gguf.get_tensor_name_map(enum, n_layers)
    out = {}
    for name, mod in model.named_modules():
        if isinstance(mod, (nn.Linear, nn.Embedding)):
            g = nm.get_name(name)
            if g is not None:
                out[name] = g
    return out


def collect_hessians(model, batches, gguf_ne0, arch, n_layers, layer_lo=0, layer_hi=None,
                     progress_every=16, log=print):
    """Same contract as coldpress.hessians.collect_hessians; X^T X accumulates on the device.

    Returns ({gguf_name: {"H": float32 [d, d] numpy, "n": int}}, unmapped)."""
    import torch
    import torch.nn as nn
    if layer_hi is None:
        layer_hi = n_layers
    name_map = build_name_map(model, arch, n_layers)
    acc, cnt = {}, {}
    unmapped, mismatched, plan = [], [], []
    for mname, mod in model.named_modules():
        if not isinstance(mod, (nn.Linear, nn.Embedding)):
            continue
        base = name_map.get(mname)
        if base is None:
            unmapped.append(mname)
            continue
        gname = base + ".weight"
        if gname not in gguf_ne0:
            unmapped.append(mname + f" (->{gname}, absent from GGUF)")
            continue
        blk = _block_index(gname)
        in_shard = (layer_lo <= blk < layer_hi) if blk >= 0 else (layer_lo == 0)
        if not in_shard:
            continue
        if isinstance(mod, nn.Linear) and mod.in_features != gguf_ne0[gname]:
            mismatched.append((mname, gname, mod.in_features, gguf_ne0[gname]))
            continue
        plan.append((mod, gname))
    if mismatched:
        for mname, gname, inf, ne0 in mismatched:
            log(f"  SHAPE MISMATCH {mname} -> {gname}: in_features={inf} ne0={ne0}")
        raise ValueError(f"{len(mismatched)} module(s) map to a GGUF tensor with a "
                         f"different ne[0]; refusing to mis-key a Hessian (see log above)")

    def make_hook(gname):
        def fn(mod, inp, out):
            x = inp[0]
            if not torch.is_floating_point(x):
                return
            x = x.detach().reshape(-1, x.shape[-1])
            if not x.is_cuda:
                raise nat.CudaPathError("collect_hessians(device CUDA): activations must be on a CUDA device")
            d = x.shape[1]
            if gname not in acc:
                acc[gname] = torch.zeros(d, d, dtype=torch.float32, device=x.device)
                cnt[gname] = 0
            xb = x.to(torch.bfloat16).contiguous()
            if d % 128:
                raise ValueError(f"{gname}: in_features {d} is not a multiple of 128")
            xtx_accumulate(xb, acc[gname])
            cnt[gname] += x.shape[0]
        return fn

    handles = [mod.register_forward_hook(make_hook(gname)) for mod, gname in plan]
    log(f"hooked {len(handles)} matmuls in layers [{layer_lo},{layer_hi}); "
        f"{len(unmapped)} module(s) unmapped/skipped")
    try:
        with torch.inference_mode():
            for c, ids in enumerate(batches):
                if ids.dim() == 1:
                    ids = ids.unsqueeze(0)
                model(ids.to(next(model.parameters()).device))
                if progress_every and (c + 1) % progress_every == 0:
                    log(f"  chunk {c + 1}")
    finally:
        for h in handles:
            h.remove()
    hessians = {}
    for gname, H in acc.items():
        Hn = H.cpu().numpy().astype(np.float32)
        if gname in gguf_ne0 and Hn.shape[0] != gguf_ne0[gname]:
            raise ValueError(f"{gname}: collected H.shape[0]={Hn.shape[0]} != ne0={gguf_ne0[gname]}")
        hessians[gname] = {"H": Hn, "n": int(cnt[gname])}
    return hessians, unmapped
