"""GPU error-feedback (EF) encoder with the interface of coldpress/ef.py.

    from perm_b200 import ef
    raw, recon = ef.ef_encode(x, "Q2_K", qw, H, n_iter=2, damp=0.01, act_order=True)
    U = ef.cholesky_inv_upper(H, damp=0.01)

Same arguments, return types and exceptions as the reference (ef.py:46-84, 179-218); the
work runs in libcoldpress_cuda.so on the current CUDA device:
  * act-order permutation: np.argsort(-np.diag(H)) on the host, exactly the reference call,
    so ties break identically;
  * U: FP64 Cholesky of the reversed, permuted, damped H plus an FP64 triangular inverse,
    cast to float32 (the same matrix as the reference's inv-then-cholesky);
  * damping escalation x10 on a non-positive pivot, up to _max_tries (ef.py:67-76);
  * n_iter rounds of {grid commit by the k-quant fitter, ordered column sweep, repack}.
"""
import sys

import numpy as np

from . import _native as nat
from . import kquant as kq
from ._native import TYPE_ID

F32 = np.float32


def _mean_diag(Hp_diag):
    return float(np.mean(Hp_diag))


def _factor_dev(torch, H_dev, order_dev, n, shift, out_f64, stream=None, workspace=None, status=None):
    """One factorisation attempt; returns (U or None, workspace, status tensor)."""
    L = nat.lib()
    ws_bytes = L.cp_factor_workspace_bytes(n)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=H_dev.device)
    if status is None:
        status = torch.zeros(1, dtype=torch.int32, device=H_dev.device)
    U = torch.empty((n, n), dtype=torch.float64 if out_f64 else torch.float32, device=H_dev.device)
    fn = L.cp_factor_u_f64 if out_f64 else L.cp_factor_u
    nat.check(fn(nat.ptr(H_dev), n, nat.ptr(order_dev), float(shift), nat.ptr(U), nat.ptr(workspace), ws_bytes,
                 nat.ptr(status), nat.stream_ptr(torch, stream)), "cholesky_inv_upper")
    return U, workspace, status


def factor_u_dev(H_dev, order, damp=0.01, _max_tries=6, out_f64=False, diag_host=None, stream=None, log=None):
    """U factor of H[order][:, order] on the device with the reference's escalation loop.

    H_dev: torch float64 CUDA [n, n]; order: int array [n] (host).  diag_host: the host
    diagonal of H, if already known (saves a device read).  Returns (U, damp_used)."""
    torch = nat.torch_cuda()
    n = int(H_dev.shape[0])
    order = np.asarray(order, dtype=np.int64)
    if diag_host is None:
        diag_host = torch.diagonal(H_dev).cpu().numpy()
    mean_diag = _mean_diag(np.asarray(diag_host, np.float64)[order])
    base = mean_diag if mean_diag > 0.0 else 1.0
    order_dev = torch.from_numpy(order.astype(np.int32)).to(H_dev.device)
    d = damp
    ws = st = None
    for attempt in range(_max_tries):
        U, ws, st = _factor_dev(torch, H_dev, order_dev, n, d * base + 1e-8, out_f64, stream, ws, st)
        if int(st.item()) == 0:
            if attempt:
                print(f"[ef] cholesky_inv_upper: damp escalated {damp:g} -> {d:g} in "
                      f"{attempt} step(s) for a borderline Hessian (n={n})", file=sys.stderr, flush=True)
            return U, d
        d *= 10.0
    raise np.linalg.LinAlgError(
        f"cholesky_inv_upper: inv(H) not positive definite even after escalating damp to "
        f"{d / 10.0:g} (n={n}); Hessian appears degenerate")


def cholesky_inv_upper(H, damp=0.01, _max_tries=6):
    """ef.py:46-84: U = chol(inv(H + (damp*mean(diag H) + 1e-8) I)).T, float64 [n, n]."""
    torch = nat.torch_cuda()
    H = np.asarray(H)
    n = H.shape[0]
    if n % 64:
        raise ValueError(f"cholesky_inv_upper: n={n} must be a multiple of 64 on the CUDA path")
    H_dev = torch.from_numpy(np.ascontiguousarray(H, dtype=np.float64)).cuda()
    U, _ = factor_u_dev(H_dev, np.arange(n), damp, _max_tries, out_f64=True, diag_host=np.diag(H))
    return np.ascontiguousarray(U.cpu().numpy())


def prepare_u_dev(U_dev, stream=None):
    """Sweep layout of the float32 factor (built once per distinct Hessian)."""
    torch = nat.torch_cuda()
    n = int(U_dev.shape[0])
    L = nat.lib()
    ut2 = torch.empty(L.cp_ef_u_bytes(n) // 4, dtype=torch.float32, device=U_dev.device)
    nat.check(L.cp_ef_prepare_u(nat.ptr(U_dev), n, nat.ptr(ut2), nat.stream_ptr(torch, stream)), "prepare_u")
    return ut2


def ef_encode_dev(x_dev, ttype, qw_dev, ut2_dev, order, n_iter=2, stream=None, want_first_fit=False,
                  workspace=None, out=None):
    """Device EF given the prepared factor of H[order][:, order].  Returns (raw, first_fit)."""
    torch = nat.torch_cuda()
    if ttype not in nat.K_TYPES:
        raise ValueError(ttype)
    nrow, n = x_dev.shape
    if n % 256:
        raise ValueError(f"n_per_row {n} is not a multiple of 256")
    L = nat.lib()
    ws_bytes = L.cp_ef_workspace_bytes(TYPE_ID[ttype], nrow, n)
    if workspace is None or workspace.numel() < ws_bytes:
        workspace = torch.empty(ws_bytes, dtype=torch.uint8, device=x_dev.device)
    order_dev = order if isinstance(order, torch.Tensor) else \
        torch.from_numpy(np.asarray(order, np.int32)).to(x_dev.device)
    raw = out if out is not None else \
        torch.empty((nrow, kq.row_bytes(ttype, n)), dtype=torch.uint8, device=x_dev.device)
    first = torch.empty_like(raw) if want_first_fit else None
    nat.check(L.cp_ef_encode(TYPE_ID[ttype], nat.ptr(x_dev), nrow, n, nat.ptr(order_dev), nat.ptr(ut2_dev),
                             nat.ptr(qw_dev), int(n_iter), nat.ptr(raw), nat.ptr(first), nat.ptr(workspace),
                             workspace.numel(), nat.stream_ptr(torch, stream)), f"ef_encode[{ttype}]")
    return raw, first


def ef_encode(x, ttype, qw, H, n_iter=2, damp=0.01, act_order=True):
    """ef.py:179-218.  x: [nrow, n] f32; qw: imatrix means [n] or None; H: [n, n].
    Returns (raw bytes [nrow, row_bytes] uint8, recon [nrow, n] f32)."""
    torch = nat.torch_cuda()
    x = np.asarray(x)
    nrow, n = x.shape
    H = np.asarray(H)
    diag = np.diag(H)
    order = np.argsort(-diag) if act_order else np.arange(n)
    H_dev = torch.from_numpy(np.ascontiguousarray(H, dtype=np.float64)).cuda()
    U_dev, _ = factor_u_dev(H_dev, order, damp, diag_host=diag)
    del H_dev
    x_dev = torch.from_numpy(np.ascontiguousarray(x, dtype=F32)).cuda()
    qw_dev = None if qw is None else torch.from_numpy(
        np.ascontiguousarray(np.broadcast_to(np.asarray(qw, F32), (n,)))).cuda()
    raw, _ = ef_encode_dev(x_dev, ttype, qw_dev, prepare_u_dev(U_dev), order, n_iter)
    recon = kq.dequantize_dev(ttype, raw, n)
    return raw.cpu().numpy(), recon.cpu().numpy()
