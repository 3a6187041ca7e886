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
import contextlib
import ctypes
import os
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


@dataclass
class Deferred:
    """A run(defer=True) whose device work may still be running (Encoder.finish completes it)."""
    jobs: list
    raws: dict
    factors: dict
    pending: tuple
    stats: bool
    after_pack: object = None
    errs_dev: object = None
    errs_h: object = None
    status_h: object = None
    event: object = None


@dataclass
class StreamBatch:
    """One batch of Encoder.run_stream: its jobs, their Hessians ({key: float64 [d, d] on the
    device}) and host diagonals, optional output buffers, and the events after which the
    weights (inputs_event, as in run()) and the Hessians of each size (ready_events, as in
    factor()) are on the device.  `tag` is free for the caller."""
    jobs: list
    hessians: dict
    diags: dict = None
    outputs: dict = None
    inputs_event: object = None
    ready_events: dict = None
    tag: object = None


class Encoder:
    """Whole-model encoder.  overlap_sweeps: in run(), start each Hessian size's first-round
    sweeps as soon as that size's factors are done instead of after all of them (measured
    slower on the 0.6B model: the sweeps then slow the factor chain that gates the rest).
    factor_priority: CUDA stream priority of the factorisation streams (-1 high, 0 normal;
    high lets the latency-bound factor chain run ahead of the round-1 fits).
    column_major: give the sweep its weights, grid, codes and compensated weights column-major
    (one lane per row then reads and writes whole 128-byte segments), converting with grouped
    transposes; False keeps everything row-major."""

    def __init__(self, n_iter=2, damp=0.01, act_order=True, stream=None, log=None, overlap_sweeps=False,
                 factor_priority=-1, column_major=True, nvtx=None):
        self.torch = nat.torch_cuda()
        self.n_iter, self.damp, self.act_order = n_iter, damp, act_order
        self.overlap_sweeps, self.factor_priority = overlap_sweeps, factor_priority
        self.column_major = column_major
        self.stream = stream
        self.log = log
        # NVTX ranges around every stage's launches (fits, factor chains, grids, sweeps,
        # transposes and repacks, statistics), for nsys / ncu --nvtx; on when nvtx=True or the
        # environment sets PERM_B200_NVTX=1
        self.nvtx = nvtx if nvtx is not None else os.environ.get("PERM_B200_NVTX", "") not in ("", "0")
        self._ws = None
        self._fws = {}            # n -> factor workspaces, reused in stream order
        self._fstreams = {}       # n -> factorisation stream
        self._fstage = {}         # n -> ring of [pinned act-order staging, event of its last read]
        self._fstage_next = {}

    @contextlib.contextmanager
    def _range(self, name):
        if not self.nvtx:
            yield
            return
        self.torch.cuda.nvtx.range_push(name)
        try:
            yield
        finally:
            self.torch.cuda.nvtx.range_pop()

    # ---------------------------------------------------------------- factorisation
    def _fstream(self, n):
        """The factorisation stream of Hessian size n: every chain of that size runs on it, so
        a size's workspaces are reused in stream order from one call to the next."""
        if n not in self._fstreams:
            self._fstreams[n] = self.torch.cuda.Stream(priority=self.factor_priority)
        return self._fstreams[n]

    def _factor_ws(self, n, count):
        """Workspaces of the first `count` Hessians of size n (kept across calls)."""
        lst = self._fws.setdefault(n, [])
        while len(lst) < count:
            lst.append(self.torch.empty(nat.lib().cp_factor_workspace_bytes(n), dtype=self.torch.uint8,
                                        device="cuda"))
        return lst[:count]

    def _order_staging(self, n, count):
        """A pinned [count, n] int32 staging buffer for act orders, from a small ring per size;
        waits (host) until the kernel that read the buffer's previous contents has run."""
        ring = self._fstage.setdefault(n, [])
        i = self._fstage_next.get(n, 0)
        self._fstage_next[n] = (i + 1) % 3
        while len(ring) <= i:
            ring.append([None, None])
        buf, ev = ring[i]
        if ev is not None:
            ev.synchronize()
        if buf is None or buf.shape[0] < count:
            buf = self.torch.empty((count, n), dtype=self.torch.int32).pin_memory()
            ring[i][0] = buf
        return ring[i], buf[:count]

    def factor(self, hessians, diags=None, _max_tries=6, check=True, ready_events=None, start_event=None):
        """hessians: {key: torch float64 [d, d] on the device}; diags: {key: host diag} if known.
        Returns {key: Factor}.  All first attempts go out as one batched call (same-size
        Hessians advance through each factorisation step in a single launch); the status
        words are read with one synchronisation and only a non-positive pivot triggers the
        reference's damp escalation for that Hessian.  ready_events: {n: CUDA event} after
        which the Hessians of size n are on the device (each size's chain waits for its own
        event instead of for everything queued on this stream).  start_event: the point of
        this stream the other chains wait for (default: everything queued so far)."""
        torch = self.torch
        L = nat.lib()
        keys = sorted(hessians, key=lambda k: -int(hessians[k].shape[0]))
        if not keys:
            self._pending = (keys, None, hessians, diags, _max_tries)
            self._factor_done = {}
            return {}
        sizes = sorted({int(hessians[k].shape[0]) for k in keys}, reverse=True)
        groups = {n: [k for k in keys if int(hessians[k].shape[0]) == n] for n in sizes}
        main = self.stream if self.stream is not None else torch.cuda.current_stream()
        # each chain's first launch zeroes its status words on its own stream (a zeroing on
        # the main stream could land after a chain that already ran ahead of it)
        status = torch.empty(len(keys), dtype=torch.int32, device="cuda")
        slot = {k: i for i, k in enumerate(keys)}
        if start_event is not None:
            ready = start_event
        else:
            ready = torch.cuda.Event()
            ready.record(main)
        out = {}
        self._factor_done = {}
        # Each size group is one chain of batched steps on its own stream; the largest (the
        # critical path) is prepared and launched first, so its chain starts while the host
        # still prepares the smaller ones.
        for n in sizes:
            grp = groups[n]
            st = self._fstream(n)
            st.wait_event(ready_events[n] if ready_events is not None and n in ready_events else ready)
            sp = nat.stream_ptr(torch, st)
            wss = self._factor_ws(n, len(grp))
            entry, oh = self._order_staging(n, len(grp))
            ohn = oh.numpy()
            shifts = []
            for r, k in enumerate(grp):
                diag = diags[k] if diags is not None and k in diags else torch.diagonal(hessians[k]).cpu().numpy()
                order = np.argsort(-diag) if self.act_order else np.arange(n)
                ohn[r] = order
                mean_diag = float(np.mean(np.asarray(diag, np.float64)[order]))
                shifts.append(float(self.damp * (mean_diag if mean_diag > 0.0 else 1.0) + 1e-8))
            with torch.cuda.stream(st):
                od = torch.empty((len(grp), n), dtype=torch.int32, device="cuda")
                # U is written straight into the start of the sweep's prepared layout
                ut2g = torch.empty((len(grp), L.cp_ef_u_bytes(n) // 4), dtype=torch.float32, device="cuda")
            # the act orders leave the pinned staging row through a kernel read, not a copy
            # engine, so they never wait behind bulk uploads queued on other streams
            nat.check(L.cp_fetch_host(nat.ptr(od), oh.data_ptr(), od.numel() * 4, sp), "fetch_host")
            fetched = torch.cuda.Event()
            fetched.record(st)
            entry[1] = fetched
            for t_ in (od, ut2g):   # also read on the main stream (sweeps)
                t_.record_stream(main)
            jobs = []
            for r, k in enumerate(grp):
                U = ut2g[r, :n * n].view(n, n)
                jobs.append(nat.FactorJob(hessians[k].data_ptr(), n, od[r].data_ptr(), shifts[r], U.data_ptr(),
                                          wss[r].data_ptr(), status[slot[k]:slot[k] + 1].data_ptr()))
                out[k] = Factor(U, ohn[r].astype(np.int64), od[r], self.damp, ut2g[r])
            arr = nat.job_array(nat.FactorJob, jobs)
            with self._range(f"factor n={n} x{len(grp)}"):
                nat.check(L.cp_factor_u_batch(ctypes.cast(arr, ctypes.c_void_p), len(grp), sp), "factor_u_batch")
            for k in grp:
                nat.check(L.cp_ef_prepare_u(nat.ptr(out[k].U), n, nat.ptr(out[k].ut2), sp), "prepare_u")
            done = torch.cuda.Event()
            done.record(st)
            self._factor_done[n] = done
            if check:
                main.wait_event(done)
        self._pending = (keys, status, hessians, diags, _max_tries)
        if check:
            self.escalate(out)
        return out

    def escalate(self, factors, pending=None, st_host=None):
        """Read the status words of the last factor() call (one synchronisation) and redo, with
        the reference's damp escalation, every factorisation that hit a non-positive pivot.
        pending / st_host: the record and host status words of an earlier deferred call.
        Returns the keys whose factors changed."""
        keys, status, hessians, diags, max_tries = pending if pending is not None else self._pending
        if not keys:
            return []
        if st_host is None:
            st_host = status.cpu().numpy()
        redone = []
        for i, k in enumerate(keys):
            if st_host[i] == 0:
                continue
            order = factors[k].order
            U, d = efm.factor_u_dev(hessians[k], order, damp=self.damp * 10.0, _max_tries=max_tries - 1,
                                    diag_host=(diags or {}).get(k), stream=self.stream)
            factors[k] = Factor(U, order, factors[k].order_dev, d, efm.prepare_u_dev(U, stream=self.stream))
            redone.append(k)
        return redone

    def run(self, jobs, hessians, diags=None, stats=True, outputs=None, inputs_event=None, ready_events=None,
            after_pack=None, defer=False):
        """factor() + encode() with the factorisations overlapped with the round-1 fits: the
        factor chains start on side streams, the fits (which need no U) go first on this
        stream, and the status words are read once at the end; tensors whose Hessian needed
        damp escalation are encoded again with the escalated factor.  inputs_event: a CUDA
        event after which the weights are ready (e.g. copies on another stream), or a list of
        (event, job names) in arrival order, each group's first fits waiting only for its own
        event; the factorisations, which need only the Hessians, wait for neither.
        ready_events: as in factor().  after_pack(event, names): called as soon as the packed
        bytes of the named jobs are queued (event: recorded after them on this stream),
        before the statistics and the status read, so a caller can start copying them out;
        called again for the jobs re-encoded after a damp escalation.
        defer: return (raws, Deferred) without waiting for the device; the statistics and the
        factor status words travel to pinned host memory behind the encode, and finish()
        completes the call (escalation, statistics) later, so the host can queue the next
        batch of tensors meanwhile (run_stream)."""
        main = self.stream if self.stream is not None else self.torch.cuda.current_stream()
        start = self.torch.cuda.Event()
        start.record(main)   # the Hessians are ready at this point of the stream
        staged = None
        if isinstance(inputs_event, (list, tuple)):
            staged = inputs_event
        elif inputs_event is not None:
            main.wait_event(inputs_event)
        made = {}

        def launch_factor():
            made["f"] = self.factor(hessians, diags, check=False, ready_events=ready_events, start_event=start)
            return made["f"], self._factor_done

        # the fits go out first, then the host launches the factor chains (side streams,
        # higher priority) while the GPU already works on the fits
        raws, st = self.encode(jobs, None, stats=stats, outputs=outputs, factor_fn=launch_factor,
                               staged_inputs=staged, after_pack=after_pack, defer=defer)
        factors = made["f"] if "f" in made else launch_factor()[0]
        if defer:
            torch = self.torch
            pending = self._pending
            status = pending[1]
            d = Deferred(jobs, raws, factors, pending, stats, after_pack)
            with torch.cuda.stream(main):   # main waited for every chain before its first sweep
                if st is not None:
                    d.errs_h = torch.empty(st.shape, dtype=st.dtype).pin_memory()
                    d.errs_h.copy_(st, non_blocking=True)
                    d.errs_dev = st
                if status is not None:
                    for n in self._factor_done:   # (also when no EF job waited for a chain)
                        main.wait_event(self._factor_done[n])
                    d.status_h = torch.empty(status.shape, dtype=status.dtype).pin_memory()
                    d.status_h.copy_(status, non_blocking=True)
            d.event = torch.cuda.Event()
            d.event.record(main)
            return raws, d
        redone = set(self.escalate(factors))
        if redone:
            again = [j for j in jobs if j.mode == "EF" and j.hkey in redone]
            r2, s2 = self.encode(again, factors, stats=stats, outputs={j.name: raws[j.name] for j in again},
                                 after_pack=after_pack)
            st.update(s2)
        return raws, st

    def finish(self, d):
        """Complete a deferred run(): wait for its device work, redo (as run() does) the
        factorisations that hit a non-positive pivot and the tensors that used them, and return
        (raws, stats)."""
        d.event.synchronize()
        st = self._stats(d.jobs, d.errs_h.numpy()) if d.stats else {}
        redone = set(self.escalate(d.factors, d.pending, d.status_h.numpy() if d.status_h is not None else None))
        if redone:
            again = [j for j in d.jobs if j.mode == "EF" and j.hkey in redone]
            r2, s2 = self.encode(again, d.factors, stats=d.stats, outputs={j.name: d.raws[j.name] for j in again},
                                 after_pack=d.after_pack)
            st.update(s2)
            # the re-encoded bytes are final only once the stream reaches them; callers copy
            # the bytes out on other streams as soon as finish() returns
            done = self.torch.cuda.Event()
            done.record(self.stream if self.stream is not None else self.torch.cuda.current_stream())
            done.synchronize()
        return d.raws, st

    def run_stream(self, batches, stats=True, on_batch=None):
        """Encode a model too large for one device pass, batch by batch, with one batch in
        flight ahead of the host: batch b is queued, then batch b - 1 is finished (the host
        waits for it while the device works on b), then batch b + 1 is prepared and queued.
        Batch b + 1's Hessian decodes and factor chains, queued on their own streams while the
        device still runs batch b's sweeps, overlap them.  batches: an iterable of
        StreamBatch, produced lazily (its inputs may be decoded or uploaded when it is
        drawn).  on_batch(batch, raws, stats): called as each batch finishes.
        Returns (raws, stats) over all batches."""
        raws_all, st_all = {}, {}
        inflight = []

        def done(item):
            b, d = item
            r, st = self.finish(d)
            raws_all.update(r)
            st_all.update(st)
            if on_batch is not None:
                on_batch(b, r, st)

        for b in batches:
            _, d = self.run(b.jobs, b.hessians, b.diags, stats=stats, outputs=b.outputs,
                            inputs_event=b.inputs_event, ready_events=b.ready_events, defer=True)
            inflight.append((b, d))
            while len(inflight) > 1:
                done(inflight.pop(0))
        while inflight:
            done(inflight.pop(0))
        return raws_all, st_all

    # ---------------------------------------------------------------- tensors
    def _arena(self, jobs):
        """Per-job scratch (codes, compensated weights, grid, sweep workspace, baseline bytes),
        carved from a few flat buffers that are reused while the job shapes stay the same."""
        torch = self.torch
        L = nat.lib()
        cm = self.column_major
        # keyed by the jobs' shapes only, so successive batches of like layers share one arena
        key = (cm,) + tuple((j.ttype, j.mode, int(j.x.shape[0]), int(j.x.shape[1])) for j in jobs)
        if getattr(self, "_arena_key", None) == key:
            return self._arena_views
        sizes = {"codes": 0, "wcur": 0, "grid": 0, "work": 0, "base": 0, "xt": 0, "ct": 0, "wt": 0}
        plan = []
        for j in jobs:
            nrow, n = int(j.x.shape[0]), int(j.x.shape[1])
            ent = {}
            if j.mode == "EF":
                sbw = nat.GRID[j.ttype][0]
                R = int(L.cp_ef_sweep_rows(nrow)) if cm else nrow   # rows of the column-major layout
                ent["codes"] = (sizes["codes"], nrow * n)
                sizes["codes"] += _al(nrow * n)
                ent["wcur"] = (sizes["wcur"], nrow * n)
                sizes["wcur"] += _al(nrow * n)
                ent["dl"] = (sizes["grid"], R * (n // sbw))
                sizes["grid"] += _al(R * (n // sbw))
                ent["ml"] = (sizes["grid"], R * (n // sbw))
                sizes["grid"] += _al(R * (n // sbw))
                if cm:
                    for k in ("xt", "ct", "wt"):
                        ent[k] = (sizes[k], R * n)
                        sizes[k] += _al(R * n)
                wb = L.cp_ef_sweep_workspace_bytes(nrow, n)
                ent["work"] = (sizes["work"], wb // 4)
                sizes["work"] += _al(wb // 4)
            if j.mode == "wRTN(attn0-diag)":
                rb = nrow * kq.row_bytes(j.ttype, n)
                ent["base"] = (sizes["base"], rb)
                sizes["base"] += _al(rb)
            plan.append(ent)
        self._arena_buf = {
            "codes": torch.empty(max(1, sizes["codes"]), dtype=torch.int8, device="cuda"),
            "wcur": torch.empty(max(1, sizes["wcur"]), dtype=torch.float32, device="cuda"),
            "grid": torch.empty(max(1, sizes["grid"]), dtype=torch.float32, device="cuda"),
            "work": torch.empty(max(1, sizes["work"]), dtype=torch.float32, device="cuda"),
            "base": torch.empty(max(1, sizes["base"]), dtype=torch.uint8, device="cuda"),
            "xt": torch.empty(max(1, sizes["xt"]), dtype=torch.float32, device="cuda"),
            "ct": torch.empty(max(1, sizes["ct"]), dtype=torch.int8, device="cuda"),
            "wt": torch.empty(max(1, sizes["wt"]), dtype=torch.float32, device="cuda"),
        }
        views = []
        for j, ent in zip(jobs, plan):
            nrow, n = int(j.x.shape[0]), int(j.x.shape[1])
            v = {}
            for k, (off, cnt) in ent.items():
                src = {"codes": "codes", "wcur": "wcur", "dl": "grid", "ml": "grid", "work": "work",
                       "base": "base", "xt": "xt", "ct": "ct", "wt": "wt"}[k]
                v[k] = self._arena_buf[src][off:off + cnt]
            views.append(v)
        self._arena_key, self._arena_views = key, views
        return views

    def encode(self, jobs, factors, stats=True, outputs=None, factor_event=None, factor_fn=None,
               staged_inputs=None, after_pack=None, defer=False):
        """Encode every job with grouped launches; returns ({name: raw uint8 on device},
        {name: stats dict}).  factor_fn: called (instead of passing factors) once the first
        round's fits and grids are queued; returns (factors, factor_event).  staged_inputs:
        [(event, job names)], the weights of each group ready after its event.  after_pack:
        as in run()."""
        torch = self.torch
        L = nat.lib()
        s = nat.stream_ptr(torch, self.stream)
        views = self._arena(jobs)
        raws = []
        for j in jobs:
            nrow, n = int(j.x.shape[0]), int(j.x.shape[1])
            raw = outputs[j.name] if outputs is not None and j.name in outputs else \
                torch.empty((nrow, kq.row_bytes(j.ttype, n)), dtype=torch.uint8, device="cuda")
            raws.append(raw)
        errs = torch.zeros((len(jobs), 2), dtype=torch.float64, device="cuda")
        ef_idx = [i for i, j in enumerate(jobs) if j.mode == "EF"]

        def fit_batch(items):  # items: (type, x, qw, out)
            by_type = {}
            for tt, x, qw, out in items:
                by_type.setdefault(tt, []).append(nat.FitJob(nat.addr(x), nat.addr(qw), nat.addr(out),
                                                             int(x.shape[0]), int(x.shape[1])))
            for tt, lst in by_type.items():
                arr = nat.job_array(nat.FitJob, lst)
                with self._range(f"fit {tt} x{len(lst)}"):
                    nat.check(L.cp_kquant_encode_batch(TYPE_ID[tt], ctypes.cast(arr, ctypes.c_void_p), len(lst), s),
                              "kquant_encode_batch")

        def block_call(fn, items, what):
            if not items:
                return
            arr = nat.job_array(nat.BlockJob, items)
            with self._range(what):
                nat.check(fn(ctypes.cast(arr, ctypes.c_void_p), len(items), s), what)

        cm = self.column_major
        pitch = {i: int(L.cp_ef_sweep_rows(int(jobs[i].x.shape[0]))) for i in ef_idx} if cm else {}

        def transpose(items, what):  # items: (src, dst, rows, cols, src_ld, dst_ld, elem_bytes)
            if not items:
                return
            arr = nat.job_array(nat.TransposeJob, [nat.TransposeJob(*it) for it in items])
            with self._range(what):
                nat.check(L.cp_transpose_batch(ctypes.cast(arr, ctypes.c_void_p), len(items), s), what)

        def werr_items(idx_list, col, use_base=False):
            out = []
            for i in idx_list:
                j = jobs[i]
                src = views[i]["base"] if use_base else raws[i]
                out.append(nat.BlockJob(TYPE_ID[j.ttype], nat.addr(src), None, None, nat.addr(j.x), nat.addr(j.qw),
                                        None, None, errs[i, col].data_ptr(), int(j.x.shape[0]), int(j.x.shape[1])))
            return out

        # round 1 fits (EF from x) together with the weighted-RTN fits
        def round1_items(idx):
            items = []
            for i in idx:
                j = jobs[i]
                if j.mode == "EF":
                    items.append((j.ttype, j.x, j.qw, raws[i]))
                elif j.mode == "wRTN(attn0-diag)":
                    items.append((j.ttype, j.x, j.fit_w, raws[i]))
                    if stats:
                        items.append((j.ttype, j.x, j.qw, views[i]["base"].view(raws[i].shape)))
                elif j.mode == "wRTN":
                    items.append((j.ttype, j.x, j.qw, raws[i]))
                else:
                    raise ValueError(f"unknown mode {j.mode}")
            return items

        main = self.stream if self.stream is not None else torch.cuda.current_stream()
        if staged_inputs:
            slot = {j.name: i for i, j in enumerate(jobs)}
            left = set(range(len(jobs)))
            for ev, names in staged_inputs:
                idx = [slot[nm] for nm in names if nm in slot and slot[nm] in left]
                main.wait_event(ev)
                fit_batch(round1_items(idx))
                left.difference_update(idx)
            fit_batch(round1_items(sorted(left)))
        else:
            fit_batch(round1_items(range(len(jobs))))
        if stats:  # stock baseline = round-1 committed bytes (EF) or the separate qw fit (attn0)
            block_call(L.cp_weighted_err_batch, werr_items(ef_idx, 1), "weighted_err_batch")
            block_call(L.cp_weighted_err_batch,
                       werr_items([i for i, j in enumerate(jobs) if j.mode == "wRTN(attn0-diag)"], 1, True),
                       "weighted_err_batch")
        if cm:  # the sweep's weights column-major, once for every round
            transpose([(nat.addr(jobs[i].x), nat.addr(views[i]["xt"]), int(jobs[i].x.shape[0]),
                        int(jobs[i].x.shape[1]), int(jobs[i].x.shape[1]), pitch[i], 4) for i in ef_idx],
                      "transpose x")
        for it in range(self.n_iter):
            if it > 0:
                fit_batch([(jobs[i].ttype, views[i]["wcur"].view(jobs[i].x.shape), jobs[i].qw, raws[i])
                           for i in ef_idx])
            grid = []
            for i in ef_idx:
                j = jobs[i]
                hm = nat.GRID[j.ttype][3]
                grid.append(nat.BlockJob(TYPE_ID[j.ttype], nat.addr(raws[i]), None, None, None, None,
                                         nat.addr(views[i]["dl"]), nat.addr(views[i]["ml"]) if hm else None, None,
                                         int(j.x.shape[0]), int(j.x.shape[1]), pitch.get(i, 0)))
            block_call(L.cp_grid_params_batch, grid, "grid_params_batch")
            if it == 0 and factor_fn is not None:
                factors, factor_event = factor_fn()
            # The first round's sweeps go out per Hessian size as soon as that size's factors
            # (side streams, factor_event {n: event}) are done, smallest first, so they overlap
            # the larger factorisations; later rounds sweep everything in one launch.
            if it == 0 and factor_event and self.overlap_sweeps:
                groups = [[i for i in ef_idx if int(jobs[i].x.shape[1]) == n] for n in sorted(factor_event)]
                waits = [factor_event[n] for n in sorted(factor_event)]
                left = [i for i in ef_idx if int(jobs[i].x.shape[1]) not in factor_event]
                if left:
                    groups.append(left)
                    waits.append(None)
            else:
                groups, waits = [ef_idx], [None]
                if it == 0 and factor_event:   # every sweep of the first round needs its factor
                    for n in factor_event:
                        main.wait_event(factor_event[n])
            for grp, ev in zip(groups, waits):
                if ev is not None:
                    main.wait_event(ev)
                sw = []
                for i in sorted(grp, key=lambda i: -int(jobs[i].x.shape[1])):  # longest tiles first
                    j = jobs[i]
                    f = factors[j.hkey]
                    hm = nat.GRID[j.ttype][3]
                    last = it + 1 == self.n_iter
                    xs, cs_, ws = (("xt", "ct", "wt") if cm else ("x", "codes", "wcur"))
                    sw.append(nat.SweepJob(TYPE_ID[j.ttype], nat.addr(j.x if xs == "x" else views[i][xs]),
                                           int(j.x.shape[0]), int(j.x.shape[1]),
                                           nat.addr(f.order_dev), nat.addr(f.ut2), nat.addr(views[i]["dl"]),
                                           nat.addr(views[i]["ml"]) if hm else None, nat.addr(views[i][cs_]),
                                           None if last else nat.addr(views[i][ws]),
                                           nat.addr(views[i]["work"]), pitch.get(i, 0)))
                if sw:
                    arr = nat.job_array(nat.SweepJob, sw)
                    with self._range(f"sweep round {it + 1} x{len(sw)}"):
                        nat.check(L.cp_ef_sweep_batch(ctypes.cast(arr, ctypes.c_void_p), len(sw), s),
                                  "ef_sweep_batch")
            if it == 0 and factor_event:
                for n in factor_event:   # everything after this point needs every factor
                    main.wait_event(factor_event[n])
            if cm:  # codes (and the next round's fit input) back to storage order
                tr = []
                for i in ef_idx:
                    nrow, n = int(jobs[i].x.shape[0]), int(jobs[i].x.shape[1])
                    tr.append((nat.addr(views[i]["ct"]), nat.addr(views[i]["codes"]), n, nrow, pitch[i], n, 1))
                    if it + 1 < self.n_iter:
                        tr.append((nat.addr(views[i]["wt"]), nat.addr(views[i]["wcur"]), n, nrow, pitch[i], n, 4))
                transpose(tr, "transpose sweep outputs")
            rp = []
            for i in ef_idx:
                j = jobs[i]
                rp.append(nat.BlockJob(TYPE_ID[j.ttype], None, nat.addr(raws[i]), nat.addr(views[i]["codes"]),
                                       None, None, None, None, None, int(j.x.shape[0]), int(j.x.shape[1])))
            block_call(L.cp_kquant_repack_batch, rp, "repack_batch")
        if after_pack is not None:
            packed = torch.cuda.Event()
            packed.record(main)
            after_pack(packed, [j.name for j in jobs])
        if stats:
            block_call(L.cp_weighted_err_batch, werr_items(range(len(jobs)), 0), "weighted_err_batch")
        out = {j.name: r for j, r in zip(jobs, raws)}
        if defer:   # the caller moves errs to the host behind the work (run(defer=True))
            return out, (errs if stats else None)
        return out, (self._stats(jobs, errs.cpu().numpy()) if stats else {})

    @staticmethod
    def _stats(jobs, e):
        """encode_gguf's per-tensor statistics from the [jobs, 2] error sums (ours, stock)."""
        st = {}
        for idx, j in enumerate(jobs):
            e_ours = float(e[idx, 0])
            e_base = e_ours if j.mode == "wRTN" else float(e[idx, 1])
            st[j.name] = {"type": j.ttype, "mode": j.mode,
                          "rel_err_vs_stock": e_ours / e_base - 1 if e_base else 0.0,
                          "err": e_ours, "err_stock": e_base}
        return st


def _al(n, a=64):
    return (n + a - 1) // a * a
