"""Memory-bounded whole-model encode: the tensors of a model too large for one device pass
(a Llama-3-8B-shaped model holds 8.03 B parameters and 129 Hessians up to d = 14336) go
through Encoder.run_stream in batches of whole Hessian groups.

The Hessians stay resident in the reference's storage form (hessians.py:185-207: float16
H / hscale plus the exact float32 diagonal, a quarter of the float64 bytes) and each batch
decodes its own into float64 on a decode stream (hessians.py:225-245 arithmetic,
cp_hessian_decode) just before its factorisations need them.  Batch sizes follow a byte
budget that counts everything a batch holds on the device: its encoder scratch, its
factorisation workspaces, the decoded Hessians and the U factors (two batches are in flight
at once, so the caller budgets for two).
"""
from dataclasses import dataclass

import numpy as np

from . import _native as nat
from .encoder import StreamBatch


@dataclass
class StoredHessian:
    """One Hessian in storage form on the device."""
    h16: object          # torch float16 [d, d] (H / hscale)
    diag32: object       # torch float32 [d], the exact diagonal
    hscale: float
    diag_host: np.ndarray  # float64 [d] (= diag32), for act order and damping on the host

    @property
    def d(self):
        return int(self.h16.shape[0])


def store_hessian(torch, H):
    """float32/float64 device H -> StoredHessian, as hessians.py:185-207 writes it
    (hscale = max|H| / 32768 when that exceeds 1, else 1)."""
    H32 = H.float()
    amax = float(H32.abs().max())
    # stored as float32 (np.float32(hscale)) and divided by that float32 value
    hscale = float(np.float32(amax / 32768.0)) if amax > 32768.0 else 1.0
    h16 = (H32 / hscale).to(torch.float16) if hscale != 1.0 else H32.to(torch.float16)
    d32 = torch.diagonal(H32).contiguous()
    return StoredHessian(h16, d32, float(hscale), d32.double().cpu().numpy())


def decode(torch, sh, stream):
    """StoredHessian -> float64 [d, d] on the device, queued on `stream`."""
    d = sh.d
    with torch.cuda.stream(stream):
        H = torch.empty((d, d), dtype=torch.float64, device="cuda")
    nat.check(nat.lib().cp_hessian_decode(nat.ptr(sh.h16), nat.ptr(sh.diag32), float(sh.hscale), d, nat.ptr(H),
                                          nat.stream_ptr(torch, stream)), "hessian_decode")
    return H


def ef_bytes_per_param():
    """Device bytes of encoder scratch per EF parameter: codes 1, compensated weights 4,
    sweep errors 4, the column-major weights, codes and compensated weights 4 + 1 + 4, and
    the committed grid (about 0.5)."""
    return 18.5


def hessian_bytes(n):
    """Device bytes one Hessian of size n holds while its batch is in flight: the decoded
    float64 H, the factorisation workspace (P, T and the split-K partial tiles) and the
    prepared float32 U."""
    L = nat.lib()
    return 8 * n * n + int(L.cp_factor_workspace_bytes(n)) + int(L.cp_ef_u_bytes(n))


def plan(jobs, dims, budget_bytes):
    """Cut `jobs` (in order) into batches of at most budget_bytes of device scratch, never
    separating the jobs of one Hessian (they share its factorisation).  dims: {hkey: d}.
    Returns a list of job lists."""
    groups, order = {}, []
    for j in jobs:
        key = j.hkey if j.mode == "EF" and j.hkey is not None else ("solo", j.name)
        if key not in groups:
            groups[key] = []
            order.append(key)
        groups[key].append(j)
    batches, cur, cur_bytes = [], [], 0
    for key in order:
        g = groups[key]
        cost = sum(j.params * ef_bytes_per_param() for j in g if j.mode == "EF")
        cost += sum(j.params * 0.1 for j in g if j.mode != "EF")
        if not isinstance(key, tuple):
            cost += hessian_bytes(dims[key])
        if cur and cur_bytes + cost > budget_bytes:
            batches.append(cur)
            cur, cur_bytes = [], 0
        cur.extend(g)
        cur_bytes += cost
    if cur:
        batches.append(cur)
    return batches


def batches(torch, job_batches, stored, outputs=None, decode_stream=None):
    """Yield a StreamBatch per job list of plan(), decoding its Hessians (from `stored`,
    {hkey: StoredHessian}) on decode_stream when the batch is drawn; each size's ready event
    follows its last decode."""
    dec = decode_stream if decode_stream is not None else torch.cuda.Stream(priority=-1)
    for jobs in job_batches:
        keys = sorted({j.hkey for j in jobs if j.mode == "EF" and j.hkey is not None},
                      key=lambda k: -stored[k].d)
        # the decodes wait for nothing on the main stream (they read the resident storage form
        # and write fresh buffers), so they and the factor chains behind them run while the
        # device still works on the previous batch
        hs, diags, ready = {}, {}, {}
        for k in keys:
            hs[k] = decode(torch, stored[k], dec)
            diags[k] = stored[k].diag_host
            ev = torch.cuda.Event()
            ev.record(dec)
            ready[stored[k].d] = ev
        outs = None if outputs is None else {j.name: outputs[j.name] for j in jobs if j.name in outputs}
        yield StreamBatch(jobs, hs, diags, outs, None, ready)
