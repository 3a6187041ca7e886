"""Hessian collection on the GPU (coldpress/hessians.py:85-183).

The reference hook computes `x.float(); acc += (x.T @ x).to(cpu)` for every hooked matmul.
Here the accumulator stays on the device in float32 and each batch's X^T X is accumulated by
the library's tensor-core kernel (cp_xtx_accumulate): bf16 activations directly (products of
bf16 values are exact in float32), float32 activations split exactly into hi + lo bf16 parts
(2^-17 relative remainder).  Only the summation order differs from the reference's float32
matmul.  collect_hessians keeps the reference's name mapping, shape cross-check and return
format; matmuls that read the same input tensor in one forward pass (q/k/v, gate/up) share
one accumulation.
"""
import numpy as np

from . import _native as nat

_WS = {}   # device index -> zero-initialised uint8 workspace tensor


def _workspace(torch, dev, nbytes):
    ws = _WS.get(dev)
    if ws is None or ws.numel() < nbytes:
        if ws is not None:
            torch.cuda.current_stream(dev).synchronize()
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=dev)
        _WS[dev] = ws
    return ws


def xtx_accumulate(x, H, stream=None):
    """H += x^T x.  x: torch CUDA [T, d] (bf16 or float32; float16 is widened to float32),
    H: torch float32 CUDA [d, d].  All calls share one workspace per device, so calls on one
    device are issued from one stream."""
    torch = nat.torch_cuda()
    if not (x.is_cuda and H.is_cuda):
        raise nat.CudaPathError("xtx_accumulate: activations and H must be on a CUDA device")
    if x.dim() != 2:
        raise ValueError("xtx_accumulate expects a 2-D [T, d] activation matrix")
    if x.dtype == torch.bfloat16:
        dt = nat.CP_XTX_BF16
    else:
        if not torch.is_floating_point(x):
            raise ValueError("xtx_accumulate expects floating-point activations")
        dt = nat.CP_XTX_F32
        if x.dtype != torch.float32:
            x = x.float()
    x = x.contiguous()
    T, d = x.shape
    if H.shape != (d, d) or H.dtype != torch.float32 or not H.is_contiguous():
        raise ValueError(f"H must be a contiguous float32 [{d}, {d}]")
    L = nat.lib()
    dev = x.device.index if x.device.index is not None else torch.cuda.current_device()
    ws = _workspace(torch, dev, L.cp_xtx_workspace_bytes(dt, T, d))
    nat.check(L.cp_xtx_accumulate(dt, nat.ptr(x), T, d, nat.ptr(H), nat.ptr(ws), ws.numel(),
                                  nat.stream_ptr(torch, stream)), "xtx_accumulate")
    return H


def xtx_status(device=None, stream=None):
    """Raise CudaPathError if a bounded wait in an earlier xtx_accumulate on `device` ran out
    (that H is incomplete); synchronises the stream."""
    torch = nat.torch_cuda()
    dev = torch.cuda.current_device() if device is None else device
    ws = _WS.get(dev)
    if ws is not None:
        nat.check(nat.lib().cp_xtx_status(nat.ptr(ws), nat.stream_ptr(torch, stream)), "xtx_status")


def _block_index(gguf_name):
    """Block index of a GGUF tensor name, or -1 for embd/output/norm (hessians.py:54-61)."""
    if gguf_name.startswith("blk."):
        try:
            return int(gguf_name.split(".")[1])
        except (IndexError, ValueError):
            return -1
    return -1


def build_name_map(model, arch, n_layers):
    """{module_name: gguf_base_name} through gguf's TensorNameMap, as hessians.py:64-82."""
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
                     progress_every=16, log=print, share_inputs=True):
    """Same contract as coldpress.hessians.collect_hessians; X^T X accumulates on the device.

    Returns ({gguf_name: {"H": float32 [d, d] numpy, "n": int}}, unmapped)."""
    import torch
    import torch.nn as nn
    if layer_hi is None:
        layer_hi = n_layers
    name_map = build_name_map(model, arch, n_layers)
    acc, cnt, alias = {}, {}, {}
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

    # Matmuls that read the very same input tensor in a forward pass (q/k/v, gate/up) have
    # identical Hessians.  From the first batch on, such a matmul shares the accumulator of the
    # first one; every later batch must repeat the sharing exactly or collection stops with
    # an error (share_inputs=False then accumulates every matmul on its own).
    # (Inference tensors carry no version counter; sibling projections do not modify their
    # shared input in place.)
    seen = {}    # id(input) -> (input, gname that accumulated it), per forward
    calls = {}   # gname -> accumulations in the current forward
    checked = set()
    state = {"batch": 0}

    def make_hook(gname):
        def fn(mod, inp, out):
            x = inp[0]
            if not torch.is_floating_point(x):
                return
            hit = seen.get(id(x))
            same = hit is not None and hit[0] is x
            if gname in alias:
                src = alias[gname]
                if not (same and hit[1] == src and calls.get(src) == 1) or gname in checked:
                    raise RuntimeError(f"{gname}: input no longer shared with {src}; "
                                       f"rerun with share_inputs=False")
                checked.add(gname)
                return
            if (share_inputs and same and state["batch"] == 0 and gname not in acc
                    and calls.get(hit[1]) == 1 and hit[1] not in alias):
                alias[gname] = hit[1]
                checked.add(gname)
                return
            if calls.get(gname) and gname in alias.values():
                raise RuntimeError(f"{gname}: called twice in one forward while its accumulator is "
                                   f"shared; rerun with share_inputs=False")
            x2 = x.detach().reshape(-1, x.shape[-1])
            d = x2.shape[1]
            if gname not in acc:
                acc[gname] = torch.zeros(d, d, dtype=torch.float32, device=x2.device)
                cnt[gname] = 0
            xtx_accumulate(x2, acc[gname])
            cnt[gname] += x2.shape[0]
            calls[gname] = calls.get(gname, 0) + 1
            if not same:
                seen[id(x)] = (x, gname)
        return fn

    handles = [mod.register_forward_hook(make_hook(gname)) for mod, gname in plan]
    log(f"hooked {len(handles)} matmuls in layers [{layer_lo},{layer_hi}); "
        f"{len(unmapped)} module(s) unmapped/skipped")
    try:
        with torch.inference_mode():
            for c, ids in enumerate(batches):
                if ids.dim() == 1:
                    ids = ids.unsqueeze(0)
                seen.clear()
                calls.clear()
                checked.clear()
                model(ids.to(next(model.parameters()).device))
                for b, a in alias.items():
                    if (b in checked) != bool(calls.get(a)):
                        raise RuntimeError(f"{b}: input no longer shared with {a}; "
                                           f"rerun with share_inputs=False")
                state["batch"] += 1
                if progress_every and (c + 1) % progress_every == 0:
                    log(f"  chunk {c + 1}")
    finally:
        seen.clear()
        for h in handles:
            h.remove()
    for dev in {H.device.index for H in acc.values() if H.is_cuda}:
        xtx_status(dev)
    for gname, first in alias.items():
        acc[gname], cnt[gname] = acc[first].clone(), cnt[first]
    hessians = {}
    for gname, H in acc.items():
        Hn = H.cpu().numpy().astype(np.float32)
        if gname in gguf_ne0 and Hn.shape[0] != gguf_ne0[gname]:
            raise ValueError(f"{gname}: collected H.shape[0]={Hn.shape[0]} != ne0={gguf_ne0[gname]}")
        hessians[gname] = {"H": Hn, "n": int(cnt[gname])}
    return hessians, unmapped
