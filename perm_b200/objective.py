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


def _as_index(torch, p, dev):
    return p.to(device=dev, dtype=torch.long) if isinstance(p, torch.Tensor) else \
        torch.as_tensor(np.asarray(p, dtype=np.int64), device=dev)


def _as_f32(torch, a, dev):
    return a.to(device=dev, dtype=torch.float32) if isinstance(a, torch.Tensor) else \
        torch.as_tensor(np.asarray(a, dtype=np.float32), device=dev)


def tensor_err(x, ttype, qw, perm=None, wvec=None, rows_sample=None, seed=0):
    """Weighted quant error of x under permutation `perm` at container `ttype`
    (objective.py:17-39): float types give 0.0, rows_sample draws the same rows as the
    reference (numpy default_rng(seed).choice, sorted)."""
    if ttype in ("F16", "F32", "BF16"):
        return 0.0
    torch = nat.torch_cuda()
    dev = "cuda"
    nrow = int(x.shape[0])
    if rows_sample and nrow > rows_sample:
        rng = np.random.default_rng(seed)
        idx = np.sort(rng.choice(nrow, rows_sample, replace=False))
        if isinstance(x, torch.Tensor):
            x = x.index_select(0, torch.as_tensor(idx, device=x.device))
        else:
            x = np.asarray(x)[idx]
    xd = _as_f32(torch, x, dev)
    qd = None if qw is None else _as_f32(torch, qw, dev)
    if perm is not None:
        pi = _as_index(torch, perm, dev)
        xd = xd.index_select(1, pi)
        qd = qd.index_select(0, pi) if qd is not None else None
    xd = xd.contiguous()
    if ttype not in kq.QUANTIZE:
        raise ValueError(f"no encoder for {ttype}")
    recon = kq.roundtrip(xd, ttype, qd)
    colerr = ((recon.double() - xd.double()) ** 2).sum(0)
    if wvec is not None:   # float64, as numpy promotes it (exact for float32 inputs)
        w = wvec.to(device=dev, dtype=torch.float64) if isinstance(wvec, torch.Tensor) else \
            torch.as_tensor(np.asarray(wvec, dtype=np.float64), device=dev)
        if perm is not None:
            w = w.index_select(0, _as_index(torch, perm, dev))
        return float((colerr * w).sum())
    if qd is not None:
        return float((colerr * qd.double()).sum())
    return float(colerr.sum())


def col_log_rms(x, row_step=32768):
    """Per-column log-RMS profile (objective.py:42-49): float64 sums of squares in row chunks."""
    torch = nat.torch_cuda()
    nrow = int(x.shape[0])
    acc = torch.zeros(int(x.shape[1]), dtype=torch.float64, device="cuda")
    for r0 in range(0, nrow, row_step):
        xc = x[r0:r0 + row_step]
        xc = xc.to(device="cuda", dtype=torch.float64) if isinstance(xc, torch.Tensor) else \
            torch.as_tensor(np.asarray(xc, dtype=np.float64), device="cuda")
        acc += (xc ** 2).sum(0)
    out = torch.log(torch.sqrt(acc / nrow) + 1e-12)
    return out.cpu().numpy() if not isinstance(x, torch.Tensor) else out
