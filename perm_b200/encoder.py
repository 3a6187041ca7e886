"""Whole-model encode on one GPU: the device pipeline behind encode_gguf(device="cuda")
(coldpress/ef.py:223-317).

Per tensor the reference chooses (ef.py:278-297):
  * "EF"                 ef_encode(x, type, qw, H) with the tensor's input Hessian;
  * "wRTN(attn0-diag)"   token_embd: QUANTIZE(x, diag(H_blk0_attn_q) / n0);
  * "wRTN"               QUANTIZE(x, qw) when no Hessian exists;
and always computes the stock baseline roundtrip(x, type, qw) for the statistics
(ef.py:298-305).  Here every step runs on the device:
  * each distinct Hessian is factorised once (q/k/v and gate/up share theirs); all first
    attempts are enqueued back to back and their status words read with one sync, and only
    a non-positive pivot triggers the reference's damp escalation;
  * EF's first committed grid is QUANTIZE(x, qw) itself, so it doubles as the stock baseline
    and the stats need no extra fit;
  * the weighted squared errors are reduced on the device; one device-to-host copy at the end.
"""
from dataclasses import dataclass

import numpy as np

from . import _native as nat
from . import ef as efm
from . import kquant as kq
from ._native import TYPE_ID


@dataclass
class Job:
    name: str
    ttype: str
    mode: str                 # "EF", "wRTN", "wRTN(attn0-diag)"
    x: object                 # torch float32 [nrow, n] on the device
    qw: object = None         # imatrix means [n] (None: reference path and unit stats weights)
    hkey: str = None          # Hessian key of an EF job
    fit_w: object = None      # column weights of the attn0-diag fit

    @property
    def params(self):
        return int(self.x.shape[0]) * int(self.x.shape[1])


@dataclass
class Factor:
    U: object                 # torch float32 [n, n] upper, the float32 cast ef_encode uses
    order: np.ndarray         # act-order permutation (host)
    order_dev: object         # int32 on the device
    damp: float
    ut2: object = None        # sweep layout of U (cp_ef_prepare_u)


class Encoder:
    def __init__(self, n_iter=2, damp=0.01, act_order=True, stream=None, log=None):
        self.torch = nat.torch_cuda()
        self.n_iter, self.damp, self.act_order = n_iter, damp, act_order
        self.stream = stream
        self.log = log
        self._ws = None
        self._fws = None
        self._fstatus = None

    # ---------------------------------------------------------------- factorisation
    def factor(self, hessians, diags=None, _max_tries=6):
        """hessians: {key: torch float64 [d, d] on the device}; diags: {key: host diag} if known.
        Returns {key: Factor}."""
        torch = self.torch
        L = nat.lib()
        keys = list(hessians)
        pending = {}
        for k in keys:
            H = hessians[k]
            n = int(H.shape[0])
            diag = diags[k] if diags is not None and k in diags else torch.diagonal(H).cpu().numpy()
            order = np.argsort(-diag) if self.act_order else np.arange(n)
            mean_diag = float(np.mean(np.asarray(diag, np.float64)[order]))
            base = mean_diag if mean_diag > 0.0 else 1.0
            pending[k] = (order, base)
        ws_bytes = max(L.cp_factor_workspace_bytes(int(hessians[k].shape[0])) for k in keys) if keys else 0
        if self._fws is None or self._fws.numel() < ws_bytes:
            self._fws = torch.empty(ws_bytes, dtype=torch.uint8, device="cuda")
        # one status word per key; the shared workspace serialises the factorisations on the stream
        status = torch.zeros(max(1, len(keys)), dtype=torch.int32, device="cuda")
        out, dev_orders = {}, {}
        for i, k in enumerate(keys):
            order, base = pending[k]
            n = len(order)
            od = torch.from_numpy(order.astype(np.int32)).to("cuda")
            dev_orders[k] = od
            U = torch.empty((n, n), dtype=torch.float32, device="cuda")
            nat.check(L.cp_factor_u(nat.ptr(hessians[k]), n, nat.ptr(od), float(self.damp * base + 1e-8), nat.ptr(U),
                                    nat.ptr(self._fws), ws_bytes, nat.ptr(status[i:i + 1]),
                                    nat.stream_ptr(torch, self.stream)), f"factor[{k}]")
            out[k] = Factor(U, order, od, self.damp)
        st = status.cpu().numpy() if keys else np.zeros(0)
        for i, k in enumerate(keys):
            if st[i] == 0:
                continue
            order, _ = pending[k]
            U, d = efm.factor_u_dev(hessians[k], order, damp=self.damp * 10.0, _max_tries=_max_tries - 1,
                                    diag_host=(diags or {}).get(k), stream=self.stream)
            out[k] = Factor(U, order, dev_orders[k], d)
        for k in keys:
            out[k].ut2 = efm.prepare_u_dev(out[k].U, stream=self.stream)
        return out

    # ---------------------------------------------------------------- tensors
    def _workspace(self, nbytes):
        if self._ws is None or self._ws.numel() < nbytes:
            self._ws = self.torch.empty(nbytes, dtype=self.torch.uint8, device="cuda")
        return self._ws

    def encode(self, jobs, factors, stats=True, outputs=None):
        """Encode every job; returns ({name: raw uint8 on device}, {name: stats dict})."""
        torch = self.torch
        L = nat.lib()
        s = nat.stream_ptr(torch, self.stream)
        ws_need = 0
        for j in jobs:
            if j.mode == "EF":
                ws_need = max(ws_need, L.cp_ef_workspace_bytes(TYPE_ID[j.ttype], j.x.shape[0], j.x.shape[1]))
        ws = self._workspace(ws_need) if ws_need else None
        errs = torch.zeros((len(jobs), 2), dtype=torch.float64, device="cuda")
        raws, bases = {}, {}
        for idx, j in enumerate(jobs):
            nrow, n = int(j.x.shape[0]), int(j.x.shape[1])
            raw = outputs[j.name] if outputs is not None and j.name in outputs else \
                torch.empty((nrow, kq.row_bytes(j.ttype, n)), dtype=torch.uint8, device="cuda")
            base = None
            if j.mode == "EF":
                f = factors[j.hkey]
                first = torch.empty_like(raw) if stats else None
                nat.check(L.cp_ef_encode(TYPE_ID[j.ttype], nat.ptr(j.x), nrow, n, nat.ptr(f.order_dev), nat.ptr(f.ut2),
                                         nat.ptr(j.qw), int(self.n_iter), nat.ptr(raw), nat.ptr(first), nat.ptr(ws),
                                         ws.numel(), s), f"ef_encode[{j.name}]")
                base = first
            elif j.mode == "wRTN(attn0-diag)":
                kq.quantize_dev(j.ttype, j.x, j.fit_w, out=raw, stream=self.stream)
                if stats:
                    base = kq.quantize_dev(j.ttype, j.x, j.qw, stream=self.stream)
            elif j.mode == "wRTN":
                kq.quantize_dev(j.ttype, j.x, j.qw, out=raw, stream=self.stream)
                base = raw
            else:
                raise ValueError(f"unknown mode {j.mode}")
            if stats:
                nat.check(L.cp_weighted_err(TYPE_ID[j.ttype], nat.ptr(raw), nat.ptr(j.x), nat.ptr(j.qw), nrow, n,
                                            nat.ptr(errs[idx, 0:1]), s), "weighted_err")
                if base is raw:
                    errs[idx, 1:2].copy_(errs[idx, 0:1])
                else:
                    nat.check(L.cp_weighted_err(TYPE_ID[j.ttype], nat.ptr(base), nat.ptr(j.x), nat.ptr(j.qw), nrow, n,
                                                nat.ptr(errs[idx, 1:2]), s), "weighted_err")
            raws[j.name] = raw
        st = {}
        if stats:
            e = errs.cpu().numpy()
            for idx, j in enumerate(jobs):
                e_ours, e_base = float(e[idx, 0]), float(e[idx, 1])
                st[j.name] = {"type": j.ttype, "mode": j.mode,
                              "rel_err_vs_stock": e_ours / e_base - 1 if e_base else 0.0}
        return raws, st
