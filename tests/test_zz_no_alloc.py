"""cp_ef_sweep_noalloc: the error-feedback sweep for callers that cannot allocate device memory
(their device memory belongs to another allocator, or they reach the library through an FFI
that cannot hand it a scratch buffer).  It keeps its per-row errors in a fixed array inside the
library.  Checked through the C ABI against cp_ef_sweep, which takes a caller workspace: two
calls in a row with different shapes and types must both give identical codes and
compensated weights, the codes must also equal the CPU oracle's sweep (coldpress/ef.py:197-216
restated) on sampled rows, and an oversized shape must be refused.

This file is named so that pytest collects it last."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _inputs(torch, nat, tt, nrow, n, seed):
    from perm_b200 import ef, kquant as kq
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    X = torch.randn(2048, n, device="cuda", dtype=torch.float64, generator=g)
    X *= torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
    H = X.T @ X / 2048
    diag = torch.diagonal(H).cpu().numpy()
    order = np.argsort(-diag)
    U, _ = ef.factor_u_dev(H, order, 0.01, diag_host=diag)
    ut2 = ef.prepare_u_dev(U)
    x = torch.randn(nrow, n, device="cuda", generator=g, dtype=torch.float32) * 0.02
    qw = torch.from_numpy(diag.astype(np.float32)).cuda()
    raw = kq.quantize_dev(tt, x, qw)
    dl, ml, *_ = kq.grid_params_dev(tt, raw, nrow, n)
    od = torch.from_numpy(order.astype(np.int32)).cuda()
    return x, od, U, ut2, dl, ml, order


def _sweep(torch, nat, tt, x, od, ut2, dl, ml, noalloc):
    L = nat.lib()
    nrow, n = x.shape
    codes = torch.full((nrow, n), 99, dtype=torch.int8, device="cuda")
    w_out = torch.full((nrow, n), float("nan"), dtype=torch.float32, device="cuda")
    s = nat.stream_ptr(torch)
    if noalloc:
        rc = L.cp_ef_sweep_noalloc(nat.TYPE_ID[tt], nat.ptr(x), nrow, n, nat.ptr(od), nat.ptr(ut2), nat.ptr(dl),
                                   nat.ptr(ml), nat.ptr(codes), nat.ptr(w_out), s)
    else:
        ws = torch.empty(L.cp_ef_sweep_workspace_bytes(nrow, n), dtype=torch.uint8, device="cuda")
        rc = L.cp_ef_sweep(nat.TYPE_ID[tt], nat.ptr(x), nrow, n, nat.ptr(od), nat.ptr(ut2), nat.ptr(dl), nat.ptr(ml),
                           nat.ptr(codes), nat.ptr(w_out), nat.ptr(ws), ws.numel(), s)
    assert rc == nat.CP_OK, nat.last_error()
    torch.cuda.synchronize()
    return codes.cpu().numpy(), w_out.cpu().numpy()


def test_noalloc_sweep_matches_workspace_sweep_twice():
    import torch
    from perm_b200 import _native as nat
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    # two calls in a row, different types and shapes: the second must not see the first's
    # leftovers in the shared scratch
    from oracle import oracle as orc
    for tt, nrow, n, seed in (("Q2_K", 3000, 1024, 1), ("Q3_K", 1000, 2048, 2)):
        x, od, U, ut2, dl, ml, order = _inputs(torch, nat, tt, nrow, n, seed)
        ml = ml if nat.GRID[tt][3] else None
        want_codes, want_w = _sweep(torch, nat, tt, x, od, ut2, dl, ml, noalloc=False)
        got_codes, got_w = _sweep(torch, nat, tt, x, od, ut2, dl, ml, noalloc=True)
        assert np.array_equal(got_codes, want_codes), f"{tt}: {np.count_nonzero(got_codes != want_codes)} codes differ"
        assert np.array_equal(got_w.view(np.int32), want_w.view(np.int32)), f"{tt}: compensated weights differ"
        # the same rows through the oracle's sweep, given the same U and committed grid
        rows = np.unique(np.r_[np.arange(40), np.linspace(0, nrow - 1, 24).astype(np.int64)])
        dl_h = dl.view(nrow, -1).cpu().numpy()[rows]
        ml_h = ml.view(nrow, -1).cpu().numpy()[rows] if ml is not None else np.zeros_like(dl_h)
        o_codes, _ = orc.ef_sweep(x.cpu().numpy()[rows], order, U.cpu().numpy(), dl_h, ml_h, tt)
        assert np.array_equal(got_codes[rows].astype(np.int32), o_codes), \
            f"{tt}: {np.count_nonzero(got_codes[rows] != o_codes)} codes differ from the oracle"


def test_noalloc_sweep_refuses_shapes_beyond_its_scratch():
    import torch
    from perm_b200 import _native as nat
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    L = nat.lib()
    nrow, n = 4128, 1024   # ceil(4128/128)*128 * 1024 * 4 bytes = 16.5 MiB > 16 MiB
    dummy = torch.zeros(16, device="cuda")
    rc = L.cp_ef_sweep_noalloc(nat.TYPE_ID["Q2_K"], nat.ptr(dummy), nrow, n, nat.ptr(dummy), nat.ptr(dummy),
                               nat.ptr(dummy), nat.ptr(dummy), nat.ptr(dummy), None, nat.stream_ptr(torch))
    assert rc == nat.CP_ERR_WORKSPACE
    assert "exceeds" in nat.last_error()
