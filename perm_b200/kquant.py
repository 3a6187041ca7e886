"""GPU k-quant codec with the interface of coldpress/kquant.py (QUANTIZE / DEQUANTIZE /
roundtrip, kquant.py:732-741).

    from perm_b200 import kquant as kq
    raw = kq.QUANTIZE["Q2_K"](x, qw)        # x: f32 [nrow, n], qw: f32 [n] or None
    y = kq.DEQUANTIZE["Q2_K"](raw, n)

numpy in, fresh numpy out (inputs are never mutated), bytes identical to the reference for
the same float32 inputs.  torch CUDA tensors are accepted too and then stay on the device.
Every call runs libcoldpress_cuda.so kernels on the current CUDA device; there is no CPU
path.
"""
import numpy as np

from . import _native as nat
from ._native import BYTES_PER_BLOCK, BLOCK_ELEMS, TYPE_ID

F32 = np.float32
QK_K = 256
BYTES_PER_SB = {t: BYTES_PER_BLOCK[t] for t in nat.K_TYPES}
SUB_W = {"Q2_K": 16, "Q3_K": 16, "Q4_K": 32, "Q5_K": 32, "Q6_K": 16}


def _check_shape(ttype, n):
    if ttype not in TYPE_ID:
        raise ValueError(ttype)
    if n % BLOCK_ELEMS[ttype]:
        if ttype == "Q2_K":  # kquant.py:351
            raise AssertionError(f"n_per_row {n} is not a multiple of {QK_K}")
        raise ValueError(f"cannot reshape a row of {n} values into {BLOCK_ELEMS[ttype]}-value blocks")


def row_bytes(ttype, n):
    return n // BLOCK_ELEMS[ttype] * BYTES_PER_BLOCK[ttype]


def quantize_dev(ttype, x, qw=None, out=None, stream=None):
    """x: torch f32 CUDA [nrow, n] (contiguous); qw: torch f32 CUDA [n] or None."""
    torch = nat.torch_cuda()
    nrow, n = x.shape
    _check_shape(ttype, n)
    if out is None:
        out = torch.empty((nrow, row_bytes(ttype, n)), dtype=torch.uint8, device=x.device)
    nat.check(nat.lib().cp_kquant_encode(TYPE_ID[ttype], nat.ptr(x), nrow, n, nat.ptr(qw), nat.ptr(out),
                                         nat.stream_ptr(torch, stream)), f"QUANTIZE[{ttype}]")
    return out


def dequantize_dev(ttype, raw, n, out=None, stream=None):
    torch = nat.torch_cuda()
    nrow = raw.shape[0]
    _check_shape(ttype, n)
    if out is None:
        out = torch.empty((nrow, n), dtype=torch.float32, device=raw.device)
    nat.check(nat.lib().cp_kquant_decode(TYPE_ID[ttype], nat.ptr(raw), nrow, n, nat.ptr(out),
                                         nat.stream_ptr(torch, stream)), f"DEQUANTIZE[{ttype}]")
    return out


def host_array(a, dtype):
    """Contiguous numpy array of `dtype` that torch.from_numpy may wrap: read-only inputs
    (np.broadcast_to views, read-only memory maps) are copied first."""
    arr = np.ascontiguousarray(a, dtype=dtype)
    return arr if arr.flags.writeable else arr.copy()


def _to_dev(torch, a, dtype):
    if isinstance(a, torch.Tensor):
        return a.to(device="cuda", dtype=dtype).contiguous()
    return torch.from_numpy(host_array(a, np.dtype(str(dtype).split(".")[-1]))).cuda()


def quantize(ttype, x, qw=None):
    torch = nat.torch_cuda()
    is_t = isinstance(x, torch.Tensor)
    xd = _to_dev(torch, x, torch.float32)
    if xd.dim() != 2:
        raise ValueError("x must be 2-D [nrow, n_per_row]")
    qd = None
    if qw is not None:
        qd = _to_dev(torch, np.broadcast_to(np.asarray(qw, F32), (xd.shape[1],)) if not isinstance(qw, torch.Tensor)
                     else qw, torch.float32)
    out = quantize_dev(ttype, xd, qd)
    return out if is_t else out.cpu().numpy()


def dequantize(ttype, raw, n):
    torch = nat.torch_cuda()
    is_t = isinstance(raw, torch.Tensor)
    rd = _to_dev(torch, raw, torch.uint8)
    out = dequantize_dev(ttype, rd, n)
    return out if is_t else out.cpu().numpy()


QUANTIZE = {t: (lambda x, qw=None, _t=t: quantize(_t, x, qw)) for t in TYPE_ID}
DEQUANTIZE = {t: (lambda raw, n_per_row, _t=t: dequantize(_t, raw, n_per_row)) for t in TYPE_ID}


def roundtrip(x, ttype, qw=None):
    """quantize then dequantize; returns the reconstruction (kquant.py:738-741)."""
    torch = nat.torch_cuda()
    is_t = isinstance(x, torch.Tensor)
    xd = _to_dev(torch, x, torch.float32)
    qd = None if qw is None else _to_dev(torch, qw, torch.float32)
    y = dequantize_dev(ttype, quantize_dev(ttype, xd, qd), xd.shape[1])
    return y if is_t else y.cpu().numpy()


def grid_params_dev(ttype, raw, nrow, n, stream=None):
    """ef.py:87-127 on the device: (dl, ml or None, lo, hi, sub-block width)."""
    torch = nat.torch_cuda()
    sbw, lo, hi, has_min = nat.GRID[ttype]
    dl = torch.empty((nrow, n // sbw), dtype=torch.float32, device=raw.device)
    ml = torch.empty_like(dl) if has_min else None
    nat.check(nat.lib().cp_grid_params(TYPE_ID[ttype], nat.ptr(raw), nrow, n, nat.ptr(dl), nat.ptr(ml),
                                       nat.stream_ptr(torch, stream)), f"grid_params[{ttype}]")
    return dl, ml, lo, hi, sbw


def codes_dev(ttype, raw, nrow, n, stream=None):
    torch = nat.torch_cuda()
    c = torch.empty((nrow, n), dtype=torch.int8, device=raw.device)
    nat.check(nat.lib().cp_kquant_codes(TYPE_ID[ttype], nat.ptr(raw), nrow, n, nat.ptr(c),
                                        nat.stream_ptr(torch, stream)), f"codes[{ttype}]")
    return c


def repack_dev(ttype, raw, codes, nrow, n, stream=None):
    """ef.py:130-176 _repack on the device, in place on `raw`."""
    torch = nat.torch_cuda()
    nat.check(nat.lib().cp_kquant_repack(TYPE_ID[ttype], nat.ptr(raw), nat.ptr(codes), nrow, n,
                                         nat.stream_ptr(torch, stream)), f"repack[{ttype}]")
    return raw
