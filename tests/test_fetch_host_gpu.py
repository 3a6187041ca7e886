"""cp_fetch_host: kernel-read copy from pinned host memory (used for the factorisation's act
orders so that they do not wait behind bulk copy-engine uploads)."""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("nbytes,offset", [(4 * 3072 * 28, 0), (1, 0), (37, 3), (4096 + 5, 16), (12345, 7)])
def test_fetch_host_copies_pinned_bytes(nbytes, offset):
    import torch
    from perm_b200 import _native as nat
    L = nat.lib()
    rng = np.random.default_rng(nbytes)
    src = torch.from_numpy(rng.integers(0, 256, nbytes + offset, dtype=np.uint8)).pin_memory()
    dst = torch.zeros(nbytes + offset, dtype=torch.uint8, device="cuda")
    s = nat.stream_ptr(torch, torch.cuda.current_stream())
    nat.check(L.cp_fetch_host(ctypes.c_void_p(dst.data_ptr() + offset), ctypes.c_void_p(src.data_ptr() + offset),
                              nbytes, s), "fetch_host")
    got = dst.cpu().numpy()
    assert np.array_equal(got[offset:], src.numpy()[offset:])
    assert not got[:offset].any()


def test_fetch_host_rejects_pageable_memory():
    import torch
    from perm_b200 import _native as nat
    L = nat.lib()
    src = np.arange(64, dtype=np.uint8)          # ordinary (pageable) host memory
    dst = torch.zeros(64, dtype=torch.uint8, device="cuda")
    s = nat.stream_ptr(torch, torch.cuda.current_stream())
    rc = L.cp_fetch_host(ctypes.c_void_p(dst.data_ptr()), ctypes.c_void_p(src.ctypes.data), 64, s)
    assert rc == nat.CP_ERR_ARG
    assert not dst.cpu().numpy().any()
