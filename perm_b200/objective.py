"""Device PERM objective with the interface of coldpress/perm/objective.py:17-51.

    from perm_b200 import objective
    err = objective.tensor_err(x, "Q2_K", qw, perm=P)

err(P) = sum_c w[c] * sum_r (x_hat[r, c] - x[r, c])^2 on x[:, P] (w = wvec[P], else qw[P],
else 1), where x_hat is the k-quant roundtrip at the tensor's target type: the quantize and
dequantize kernels of libcoldpress_cuda.so, byte-identical to coldpress.kquant, so x_hat is
the reference's reconstruction exactly.  The squared differences and sums are float64 as in
the reference (objective.py:31-39); only the summation order differs (float64 rounding).
x, qw, perm and wvec may be numpy arrays or torch tensors (CUDA tensors stay on the device).
"""
import numpy as np

from . import _native as nat
from . import kquant as kq


def _dev_f32(torch, a):
    """float32 CUDA tensor (contiguous) of a numpy array or tensor."""
    if isinstance(a, torch.Tensor):
        return a.to(device="cuda", dtype=torch.float32).contiguous()
    return torch.from_numpy(kq.host_array(a, np.float32)).cuda()


def _dev_index(torch, p):
    if p is None:
        return None
    if isinstance(p, torch.Tensor):
        return p.to(device="cuda", dtype=torch.int64).contiguous()
    return torch.from_numpy(kq.host_array(p, np.int64)).cuda()


def _gather(torch, src, ld, rows, nrow_out, cols, n_out):
    out = torch.empty((nrow_out, n_out), dtype=torch.float32, device="cuda")
    nat.check(nat.lib().cp_gather_f32(nat.ptr(src), ld, nat.ptr(rows), nrow_out, nat.ptr(cols), n_out,
                                      nat.ptr(out), nat.stream_ptr(torch)), "gather_f32")
    return out


def _host_f64(torch, a):
    if isinstance(a, torch.Tensor):
        return a.detach().to("cpu", torch.float64).numpy()
    return np.asarray(a, dtype=np.float64)


def tensor_err(x, ttype, qw, perm=None, wvec=None, rows_sample=None, seed=0):
    """Weighted quant error of x under permutation `perm` at container `ttype`
    (objective.py:17-39): float types give 0.0, rows_sample draws the same rows as the
    reference (numpy default_rng(seed).choice, sorted).  On the device: one gather kernel
    (row sample and column permutation), the quantize and dequantize kernels, and one
    per-column float64 squared-error kernel; the host finishes with the reference's own
    float64 dot product of the n column errors with the weights."""
    if ttype in ("F16", "F32", "BF16"):
        return 0.0
    if ttype not in kq.QUANTIZE:
        raise ValueError(f"no encoder for {ttype}")
    torch = nat.torch_cuda()
    xd = _dev_f32(torch, x)
    if xd.dim() != 2:
        raise ValueError("x must be 2-D [nrow, n_per_row]")
    nrow, n = int(xd.shape[0]), int(xd.shape[1])
    rows = None
    if rows_sample and nrow > rows_sample:
        rng = np.random.default_rng(seed)
        rows = _dev_index(torch, np.sort(rng.choice(nrow, rows_sample, replace=False)))
    pi = _dev_index(torch, perm)
    if rows is not None or pi is not None:
        xd = _gather(torch, xd, n, rows, int(rows.numel()) if rows is not None else nrow, pi, n)
    qd = None
    if qw is not None:
        qd = _dev_f32(torch, qw)
        if pi is not None:
            qd = _gather(torch, qd, n, None, 1, pi, n).view(n)
    raw = kq.quantize_dev(ttype, xd, qd)
    recon = kq.dequantize_dev(ttype, raw, n)
    colerr = torch.empty(n, dtype=torch.float64, device="cuda")
    nat.check(nat.lib().cp_col_sqdiff(nat.ptr(recon), nat.ptr(xd), int(xd.shape[0]), n, n, nat.ptr(colerr),
                                      nat.stream_ptr(torch)), "col_sqdiff")
    colerr = colerr.cpu().numpy()
    p_host = None if perm is None else _host_f64(torch, perm).astype(np.int64)
    if wvec is not None:   # float64, as numpy promotes it
        w = _host_f64(torch, wvec)
        return float((colerr * (w[p_host] if p_host is not None else w)).sum())
    if qd is not None:
        return float((colerr * qd.cpu().numpy().astype(np.float64)).sum())
    return float(colerr.sum())


def col_log_rms(x, row_step=32768):
    """Per-column log-RMS profile (objective.py:42-49): float64 column sums of squares on the
    device (one kernel per row chunk of x when x is a host array, so only a chunk at a time
    travels), then the n logs on the host."""
    torch = nat.torch_cuda()
    nrow, n = int(x.shape[0]), int(x.shape[1])
    acc = np.zeros(n, np.float64)
    part = torch.empty(n, dtype=torch.float64, device="cuda")
    step = nrow if isinstance(x, torch.Tensor) else max(1, row_step)
    for r0 in range(0, nrow, step):
        xc = _dev_f32(torch, x[r0:r0 + step])
        nat.check(nat.lib().cp_col_sqdiff(nat.ptr(xc), None, int(xc.shape[0]), n, n, nat.ptr(part),
                                          nat.stream_ptr(torch)), "col_sqdiff")
        acc += part.cpu().numpy()
    out = np.log(np.sqrt(acc / nrow) + 1e-12)
    return torch.from_numpy(out).cuda() if isinstance(x, torch.Tensor) else out
