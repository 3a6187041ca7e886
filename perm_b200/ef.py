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
    H_dev = torch.from_numpy(kq.host_array(H, np.float64)).cuda()
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
    H_dev = torch.from_numpy(kq.host_array(H, np.float64)).cuda()
    U_dev, _ = factor_u_dev(H_dev, order, damp, diag_host=diag)
    del H_dev
    x_dev = torch.from_numpy(kq.host_array(x, F32)).cuda()
    qw_dev = None if qw is None else torch.from_numpy(
        kq.host_array(np.broadcast_to(np.asarray(qw, F32), (n,)), F32)).cuda()
    raw, _ = ef_encode_dev(x_dev, ttype, qw_dev, prepare_u_dev(U_dev), order, n_iter)
    recon = kq.dequantize_dev(ttype, raw, n)
    return raw.cpu().numpy(), recon.cpu().numpy()


# ---------------------------------------------------------------------------- driver

def _hessian_to_device(torch, st, perm=None):
    """Stored Hessian components -> float64 [d, d] on the device (hessians.py:225-245
    arithmetic); a permutation is applied on the host first (ef.py:289-290)."""
    from . import gguf_io
    h = st["h"]
    if perm is None and h.dtype == np.float16:
        d = h.shape[0]
        h16 = torch.from_numpy(kq.host_array(h, h.dtype).view(np.int16)).cuda()
        d32 = torch.from_numpy(kq.host_array(st["diag32"], np.float32)).cuda() if st["diag32"] is not None else None
        H = torch.empty((d, d), dtype=torch.float64, device="cuda")
        nat.check(nat.lib().cp_hessian_decode(nat.ptr(h16), nat.ptr(d32), float(st["hscale"]), d, nat.ptr(H),
                                              nat.stream_ptr(torch)), "hessian_decode")
        return H
    Hn = h.astype(np.float64)
    if st["hscale"] != 1.0:
        Hn *= st["hscale"]
    if st["diag32"] is not None:
        np.fill_diagonal(Hn, st["diag32"].astype(np.float64))
    if perm is not None:
        Hn = Hn[np.ix_(perm, perm)]
    return torch.from_numpy(kq.host_array(Hn, Hn.dtype)).cuda()


def encode_gguf(f16_path, target_path, hessdir, out_path, imatrix_path=None, perms=None, spacemap=None, dims=None,
                acknowledge_unreviewed=False, only="all", n_iter=2, unsafe_storage_order=False, device="cuda",
                log=print, max_params_per_batch=200_000_000, timings=None):
    """ef.py:223-317 on the GPU: EF-encode every quantized tensor of `target_path` with the f16
    weights of `f16_path` and the Hessians in `hessdir`, write a clone of the target with the
    new payloads to `out_path` and the per-tensor statistics to out_path + ".efstats.json".

    Same arguments, modes ("EF", "wRTN(attn0-diag)" for token_embd, "wRTN" without a
    Hessian), errors and outputs as the reference; identical Hessians are factorised once.
    Tensors go through the device in batches of at most max_params_per_batch parameters
    (Encoder.run_stream, one batch in flight ahead of the host), and the file work overlaps the
    device work: a reader thread loads the next batch's weights and Hessian files (npz
    decompression) while the device encodes the current one; the float16 weights and the
    stored-form Hessians (float16 / hscale + float32 diagonal) travel to the device in that
    form on a copy stream and are widened / decoded there; the packed bytes come back on
    their own stream as each batch finishes.  timings (a dict, optional) receives the wall
    time and its parts: read_s (reader thread), device_s (from the first batch queued to the
    last batch finished), write_s (the GGUF re-emit), bytes moved each way."""
    import concurrent.futures as cf
    import hashlib
    import json
    import os
    import time
    from gguf import GGUFReader
    from . import gguf_io
    from .encoder import Encoder, Job, StreamBatch
    t_start = time.time()
    if device is not None and not str(device).startswith("cuda"):
        raise ValueError(f"perm_b200.encode_gguf runs on CUDA devices only (device={device!r})")
    imat = gguf_io.imatrix_means(imatrix_path) if imatrix_path else {}
    f16 = {t.name: t for t in GGUFReader(f16_path).tensors}
    tr = GGUFReader(target_path)
    supported = set(kq.QUANTIZE)
    targets = [(t.name, t.tensor_type.name) for t in tr.tensors if t.tensor_type.name in supported]
    unsupported = [(t.name, t.tensor_type.name) for t in tr.tensors
                   if t.tensor_type.name not in supported and t.tensor_type.name not in ("F16", "F32", "BF16")]
    if unsupported:
        raise ValueError(f"target has types we cannot encode: {unsupported}")
    ack = {"acknowledge_unreviewed": acknowledge_unreviewed} if acknowledge_unreviewed else {}
    torch = nat.torch_cuda()
    if device is not None and ":" in str(device):
        torch.cuda.set_device(torch.device(device))

    def input_perm(name):
        if perms is None or spacemap is None:
            return None
        return spacemap.input_perm(name, perms, dims, **ack)

    plan = []
    for name, tt in targets:
        is_embdout = name in ("token_embd.weight", "output.weight")
        if (only == "blk" and is_embdout) or (only == "embdout" and not is_embdout):
            continue
        qw = imat.get(name)
        p = input_perm(name)
        if qw is not None and p is not None:
            qw = qw[p]
        if name == "token_embd.weight":
            H0, n0 = gguf_io.load_hessian(hessdir, "blk.0.attn_q.weight")
            fit_w = (np.diag(H0) / max(n0, 1)).astype(np.float32)
            if p is not None:
                fit_w = fit_w[p]
            plan.append((name, tt, "wRTN(attn0-diag)", qw, None, fit_w, p))
        elif gguf_io.has_hessian(hessdir, name):
            if tt not in nat.K_TYPES:
                raise ValueError(tt)  # ef.py:_grid_params supports the k-quants only
            plan.append((name, tt, "EF" if not unsafe_storage_order else "EF(storage-order)", qw, name, None, p))
        else:
            plan.append((name, tt, "wRTN", qw, None, None, p))

    batches, cur, total = [], [], 0
    for item in plan:
        ne = int(f16[item[0]].n_elements)
        if cur and total + ne > max_params_per_batch:
            batches.append(cur)
            cur, total = [], 0
        cur.append(item)
        total += ne
    if cur:
        batches.append(cur)

    clock = {"read_s": 0.0, "h2d_bytes": 0, "d2h_bytes": 0}

    def read_weight(name):
        a = np.asarray(f16[name].data)
        if a.dtype == np.float16:
            host = torch.empty(a.shape, dtype=torch.float16, pin_memory=True)
            host.numpy()[...] = a
        else:
            host = torch.empty(a.shape, dtype=torch.float32, pin_memory=True)
            host.numpy()[...] = a.astype(np.float32)
        return host

    def read_hessian(item):
        name, tt, mode, qw, hname, fit_w, p = item
        st = gguf_io.load_hessian_stored(hessdir, hname)   # npz decompression: releases the GIL
        dig = hashlib.sha1(st["h"].tobytes())
        dig.update(np.float64(st["hscale"]).tobytes())
        if st["diag32"] is not None:
            dig.update(st["diag32"].tobytes())
        if p is not None:
            dig.update(np.asarray(p, np.int64).tobytes())
        return dig.hexdigest(), st

    def read_batch(batch):
        """Reader thread: the batch's weights (float16 when the source holds float16) and its
        stored Hessians with a content digest each, in pinned host memory; the files of a
        batch are read and decompressed by a pool of host threads."""
        t0 = time.time()
        w = dict(zip([it[0] for it in batch], io.map(read_weight, [it[0] for it in batch])))
        items = [it for it in batch if it[4] is not None]
        hs, pinned = {}, set()
        for it, (key, st) in zip(items, io.map(read_hessian, items)):
            if it[6] is None and st["h"].dtype == np.float16 and key not in pinned:
                st["h_pinned"] = torch.from_numpy(np.ascontiguousarray(st["h"]).view(np.int16)).pin_memory()
                pinned.add(key)
            hs[it[0]] = (key, st)
        clock["read_s"] += time.time() - t0
        return w, hs

    enc = Encoder(n_iter=n_iter, act_order=not unsafe_storage_order)
    copy_s = torch.cuda.Stream()               # host -> device, in order
    work_s = torch.cuda.Stream(priority=-1)    # widening and Hessian decodes, ahead of the fits
    d2h_s = torch.cuda.Stream()
    main = torch.cuda.current_stream()
    pool = cf.ThreadPoolExecutor(max_workers=1)        # reads the next batch ahead
    io = cf.ThreadPoolExecutor(max_workers=max(1, min(16, os.cpu_count() or 1)))   # its files

    def stream_batches():
        fut = pool.submit(read_batch, batches[0])
        for bi, batch in enumerate(batches):
            w_host, hs_host = fut.result()
            if bi + 1 < len(batches):
                fut = pool.submit(read_batch, batches[bi + 1])
            t_draw = time.time()
            hess_dev, diags, ready, jobs, keep = {}, {}, {}, [], [w_host, hs_host]
            by_key = {}
            for name, (key, st) in hs_host.items():
                if key in by_key:
                    continue
                by_key[key] = st
                d = st["h"].shape[0]
                if "h_pinned" in st:
                    with torch.cuda.stream(copy_s):
                        h16 = torch.empty((d, d), dtype=torch.int16, device="cuda")
                        h16.copy_(st["h_pinned"], non_blocking=True)
                        d32 = None
                        if st["diag32"] is not None:
                            d32h = torch.from_numpy(st["diag32"]).pin_memory()
                            d32 = torch.empty(d, dtype=torch.float32, device="cuda")
                            d32.copy_(d32h, non_blocking=True)
                            keep.append(d32h)
                    arrived = torch.cuda.Event()
                    arrived.record(copy_s)
                    work_s.wait_event(arrived)
                    with torch.cuda.stream(work_s):
                        H = torch.empty((d, d), dtype=torch.float64, device="cuda")
                    nat.check(nat.lib().cp_hessian_decode(nat.ptr(h16), nat.ptr(d32), float(st["hscale"]), d,
                                                          nat.ptr(H), nat.stream_ptr(torch, work_s)), "hessian_decode")
                    for t_ in (h16, d32):
                        if t_ is not None:
                            t_.record_stream(work_s)
                    ev = torch.cuda.Event()
                    ev.record(work_s)
                    ready[d] = ev            # the last decode of this size so far
                    clock["h2d_bytes"] += d * d * 2 + (d * 4 if d32 is not None else 0)
                else:   # permuted or float32-stored Hessians: decoded on the host
                    p = next(item[6] for item in batch if item[4] is not None and hs_host[item[0]][0] == key)
                    H = _hessian_to_device(torch, st, p)
                    clock["h2d_bytes"] += H.numel() * 8
                hess_dev[key] = H
                if "h_pinned" in st:   # the decode's own diagonal, computed on the host
                    diags[key] = (st["diag32"].astype(np.float64) if st["diag32"] is not None else
                                  st["h"].diagonal().astype(np.float64) * float(st["hscale"]))
                else:
                    diags[key] = torch.diagonal(H).cpu().numpy()
            staged = []

            def upload_small(a):   # imatrix means / fit weights: pinned, on the copy stream
                if a is None:
                    return None
                h = torch.from_numpy(kq.host_array(a, np.float32)).pin_memory()
                with torch.cuda.stream(copy_s):
                    dv = torch.empty(h.shape, dtype=torch.float32, device="cuda")
                    dv.copy_(h, non_blocking=True)
                dv.record_stream(main)
                keep.append(h)
                return dv

            for name, tt, mode, qw, hname, fit_w, p in batch:
                host = w_host[name]
                qw_dev, fw_dev = upload_small(qw), upload_small(fit_w)
                with torch.cuda.stream(copy_s):
                    dev = torch.empty(host.shape, dtype=host.dtype, device="cuda")
                    dev.copy_(host, non_blocking=True)
                clock["h2d_bytes"] += host.numel() * host.element_size()
                arrived = torch.cuda.Event()
                arrived.record(copy_s)
                work_s.wait_event(arrived)
                with torch.cuda.stream(work_s):
                    x = dev.float() if dev.dtype != torch.float32 else dev
                dev.record_stream(work_s)
                x.record_stream(main)
                ev = torch.cuda.Event()
                ev.record(work_s)
                staged.append((ev, [name]))
                jobs.append(Job(name, tt, "EF" if mode.startswith("EF") else mode, x, qw_dev,
                                hs_host[name][0] if hname is not None else None, fw_dev))
            yield StreamBatch(jobs, hess_dev, diags, None, staged, ready, tag=(batch, t_draw, keep))

    replace, stats, pending = {}, {}, []
    t_last = [time.time()]

    def on_batch(b, raws, st):
        batch, t_draw, _keep = b.tag
        now = time.time()
        dt = now - max(t_draw, t_last[0])
        t_last[0] = now
        tot = sum(j.params for j in b.jobs) or 1
        for (name, tt, mode, *_), j in zip(batch, b.jobs):
            host = torch.empty(raws[name].shape, dtype=torch.uint8, pin_memory=True)
            with torch.cuda.stream(d2h_s):
                host.copy_(raws[name], non_blocking=True)
            clock["d2h_bytes"] += host.numel()
            pending.append((name, host, raws[name]))
            s_ = {"type": st[name]["type"], "mode": mode, "rel_err_vs_stock": st[name]["rel_err_vs_stock"],
                  "sec": dt * j.params / tot}
            stats[name] = s_
            k = len(stats)
            if k % 20 == 0 or name in ("token_embd.weight", "output.weight"):
                log(f"[{k}/{len(targets)}] {name} {tt} {mode} "
                    f"err-vs-stock {s_['rel_err_vs_stock'] * 100:+.1f}% ({s_['sec']:.1f}s)")

    t_dev = time.time()
    if batches:
        enc.run_stream(stream_batches(), stats=True, on_batch=on_batch)
    d2h_s.synchronize()
    pool.shutdown()
    io.shutdown()
    device_s = time.time() - t_dev
    for name, host, _dev in pending:
        replace[name] = host.numpy().reshape(-1)
    t_w = time.time()
    gguf_io.copy_gguf(target_path, out_path, replace)
    write_s = time.time() - t_w
    ordered = {name: stats[name] for name, *_ in plan if name in stats}
    if ordered:
        med = float(np.median([s["rel_err_vs_stock"] for s in ordered.values()]))
        log(f"median err-vs-stock: {med * 100:+.2f}%; total {(time.time() - t_start) / 60:.1f} min")
    with open(out_path + ".efstats.json", "w") as fh:
        json.dump(ordered, fh, indent=1)
    if timings is not None:
        timings.update({"wall_s": time.time() - t_start, "read_s": clock["read_s"], "device_s": device_s,
                        "write_s": write_s, "h2d_bytes": clock["h2d_bytes"], "d2h_bytes": clock["d2h_bytes"],
                        "batches": len(batches), "tensors": len(ordered)})
    return ordered
