"""The C ABI library loads on a machine without a GPU and exports every entry point that
include/coldpress_cuda.h declares (no compute calls here)."""
import ctypes
import os
import re

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "coldpress_cuda.h")).read()
    return sorted(set(re.findall(r"\b(cp_[a-z0-9_]+)\s*\(", src)))


def test_header_declares_the_hot_path():
    names = _declared()
    for must in ("cp_kquant_encode", "cp_kquant_decode", "cp_grid_params", "cp_kquant_repack",
                 "cp_factor_u", "cp_ef_encode", "cp_ef_sweep", "cp_xtx_accumulate", "cp_last_error"):
        assert must in names


def test_library_exports_every_declared_symbol():
    from perm_b200 import build
    path = build.build()
    lib = ctypes.CDLL(path)
    missing = [n for n in _declared() if not hasattr(lib, n)]
    assert not missing, f"not exported: {missing}"
    lib.cp_version.restype = ctypes.c_int
    assert lib.cp_version() >= 100
    lib.cp_block_bytes.restype = ctypes.c_int
    assert [lib.cp_block_bytes(t) for t in (10, 11, 12, 13, 14, 8, 99)] == [84, 110, 144, 176, 210, 34, 0]
    lib.cp_ef_workspace_bytes.restype = ctypes.c_size_t
    lib.cp_ef_workspace_bytes.argtypes = [ctypes.c_int, ctypes.c_int64, ctypes.c_int64]
    assert lib.cp_ef_workspace_bytes(10, 3072, 1024) > 3072 * 1024 * 4


def test_shape_errors_need_no_gpu():
    from perm_b200 import _native as nat
    L = nat.lib()
    rc = L.cp_kquant_encode(10, None, 4, 200, None, None, None)
    assert rc == nat.CP_ERR_SHAPE and "multiple" in nat.last_error()
    rc = L.cp_kquant_encode(99, None, 4, 256, None, None, None)
    assert rc == nat.CP_ERR_TYPE


def test_xtx_inject_stall_checks_its_arguments():
    from perm_b200 import _native as nat
    L = nat.lib()
    assert L.cp_xtx_inject_stall(-1, 2_000_000) == nat.CP_ERR_ARG
    assert L.cp_xtx_inject_stall(0, 10) == nat.CP_ERR_ARG
    assert L.cp_xtx_inject_stall(0, 5_000_000_000) == nat.CP_ERR_ARG
