"""ctypes binding of libcoldpress_cuda.so (include/coldpress_cuda.h).

There is no CPU fallback: if the library is missing or no CUDA device is present, every call
raises.  Device memory and streams come from PyTorch; only raw pointers cross the C ABI.
"""
import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcoldpress_cuda.so")

CP_OK, CP_ERR_TYPE, CP_ERR_SHAPE, CP_ERR_NOT_PD, CP_ERR_CUDA, CP_ERR_ARG, CP_ERR_WORKSPACE, CP_ERR_TIMEOUT = range(8)
CP_XTX_BF16, CP_XTX_F32 = 0, 1

TYPE_ID = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
K_TYPES = ("Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K")
BYTES_PER_BLOCK = {"Q2_K": 84, "Q3_K": 110, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210, "Q8_0": 34}
BLOCK_ELEMS = {"Q2_K": 256, "Q3_K": 256, "Q4_K": 256, "Q5_K": 256, "Q6_K": 256, "Q8_0": 32}
# (sub-block width, code lo, code hi, has a min), coldpress/ef.py:87-127
GRID = {"Q2_K": (16, 0, 3, True), "Q3_K": (16, -4, 3, False), "Q4_K": (32, 0, 15, True),
        "Q5_K": (32, 0, 31, True), "Q6_K": (16, -32, 31, False)}


class FitJob(ctypes.Structure):
    _fields_ = [("x", ctypes.c_void_p), ("qw", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("nrow", ctypes.c_int64), ("n", ctypes.c_int64)]


class BlockJob(ctypes.Structure):
    _fields_ = [("ggml_type", ctypes.c_int), ("raw", ctypes.c_void_p), ("raw_out", ctypes.c_void_p),
                ("codes", ctypes.c_void_p), ("x", ctypes.c_void_p), ("w", ctypes.c_void_p),
                ("dl", ctypes.c_void_p), ("ml", ctypes.c_void_p), ("err", ctypes.c_void_p),
                ("nrow", ctypes.c_int64), ("n", ctypes.c_int64), ("grid_pitch", ctypes.c_int64)]


class SweepJob(ctypes.Structure):
    _fields_ = [("ggml_type", ctypes.c_int), ("x", ctypes.c_void_p), ("nrow", ctypes.c_int64),
                ("n", ctypes.c_int64), ("order", ctypes.c_void_p), ("u_prepared", ctypes.c_void_p),
                ("dl", ctypes.c_void_p), ("ml", ctypes.c_void_p), ("codes", ctypes.c_void_p),
                ("w_out", ctypes.c_void_p), ("workspace", ctypes.c_void_p), ("pitch", ctypes.c_int64)]


class TransposeJob(ctypes.Structure):
    _fields_ = [("src", ctypes.c_void_p), ("dst", ctypes.c_void_p), ("rows", ctypes.c_int64),
                ("cols", ctypes.c_int64), ("src_ld", ctypes.c_int64), ("dst_ld", ctypes.c_int64),
                ("elem_bytes", ctypes.c_int32)]


def job_array(cls, items):
    arr = (cls * max(1, len(items)))()
    for i, it in enumerate(items):
        arr[i] = it
    return arr


class FactorJob(ctypes.Structure):
    _fields_ = [("H", ctypes.c_void_p), ("n", ctypes.c_int64), ("order", ctypes.c_void_p),
                ("diag_shift", ctypes.c_double), ("U_out", ctypes.c_void_p), ("workspace", ctypes.c_void_p),
                ("status_dev", ctypes.c_void_p)]


class CudaPathError(RuntimeError):
    """A CUDA call of the encoder failed (launch error, bad argument, missing library)."""


_lib = None


def lib():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise CudaPathError(f"{LIB_PATH} is not built; run `python -m perm_b200.build` "
                            f"(the encoder has no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I64, I, D, SZ = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_double, ctypes.c_size_t
    sig = {
        "cp_version": ([], I),
        "cp_last_error": ([], ctypes.c_char_p),
        "cp_block_bytes": ([I], I),
        "cp_profile_enable": ([I], None),
        "cp_launch_count": ([], I64),
        "cp_profile_collect": ([P, P], I),
        "cp_kquant_encode": ([I, P, I64, I64, P, P, P], I),
        "cp_kquant_decode": ([I, P, I64, I64, P, P], I),
        "cp_grid_params": ([I, P, I64, I64, P, P, P], I),
        "cp_kquant_codes": ([I, P, I64, I64, P, P], I),
        "cp_kquant_repack": ([I, P, P, I64, I64, P], I),
        "cp_weighted_err": ([I, P, P, P, I64, I64, P, P], I),
        "cp_hessian_decode": ([P, P, D, I64, P, P], I),
        "cp_factor_workspace_bytes": ([I64], SZ),
        "cp_factor_u": ([P, I64, P, D, P, P, SZ, P, P], I),
        "cp_factor_u_f64": ([P, I64, P, D, P, P, SZ, P, P], I),
        "cp_ef_u_bytes": ([I64], SZ),
        "cp_ef_prepare_u": ([P, I64, P, P], I),
        "cp_ef_sweep_workspace_bytes": ([I64, I64], SZ),
        "cp_ef_sweep": ([I, P, I64, I64, P, P, P, P, P, P, P, SZ, P], I),
        "cp_ef_workspace_bytes": ([I, I64, I64], SZ),
        "cp_ef_encode": ([I, P, I64, I64, P, P, P, I, P, P, P, SZ, P], I),
        "cp_xtx_workspace_bytes": ([I, I64, I64], SZ),
        "cp_xtx_accumulate": ([I, P, I64, I64, P, P, SZ, P], I),
        "cp_xtx_status": ([P, P], I),
        "cp_xtx_inject_stall": ([I, I64], I),
        "cp_kquant_encode_batch": ([I, P, I, P], I),
        "cp_grid_params_batch": ([P, I, P], I),
        "cp_kquant_repack_batch": ([P, I, P], I),
        "cp_weighted_err_batch": ([P, I, P], I),
        "cp_ef_sweep_batch": ([P, I, P], I),
        "cp_factor_u_batch": ([P, I, P], I),
        "cp_ef_sweep_noalloc": ([I, P, I64, I64, P, P, P, P, P, P, P], I),
        "cp_ef_sweep_rows": ([I64], I64),
        "cp_transpose_batch": ([P, I, P], I),
        "cp_fetch_host": ([P, P, I64, P], I),
        "cp_gather_f32": ([P, I64, P, I64, P, I64, P, P], I),
        "cp_col_sqdiff": ([P, P, I64, I64, I64, P, P], I),
    }
    for name, (args, res) in sig.items():
        f = getattr(L, name)
        f.argtypes = args
        f.restype = res
    _lib = L
    return L


PROFILE_CLASSES = ("fit", "sweep", "factor", "other")


def profile_enable(on=True):
    lib().cp_profile_enable(1 if on else 0)


def profile_collect():
    """{class: (ms, launches)} of the launches recorded since the last collect."""
    ms = (ctypes.c_double * 4)()
    cnt = (ctypes.c_int64 * 4)()
    check(lib().cp_profile_collect(ctypes.cast(ms, ctypes.c_void_p), ctypes.cast(cnt, ctypes.c_void_p)),
          "profile_collect")
    return {c: (ms[i], cnt[i]) for i, c in enumerate(PROFILE_CLASSES)}


def last_error():
    return lib().cp_last_error().decode(errors="replace")


def check(rc, what=""):
    if rc == CP_OK:
        return
    msg = last_error()
    if rc == CP_ERR_TYPE:
        raise ValueError(f"{what}: {msg}")
    if rc == CP_ERR_SHAPE:
        raise ValueError(f"{what}: {msg}")
    if rc == CP_ERR_NOT_PD:
        raise np.linalg.LinAlgError(f"{what}: {msg}")
    raise CudaPathError(f"{what}: status {rc}: {msg}")


def torch_cuda():
    """Import torch and require a CUDA device (the encoder has no CPU path)."""
    import torch
    if not torch.cuda.is_available():
        raise CudaPathError("coldpress CUDA encoder: no CUDA device available")
    return torch


def ptr(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def addr(t):
    """Raw device address for a job struct field (None for a missing tensor)."""
    return t.data_ptr() if t is not None else None


def stream_ptr(torch, stream=None):
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)
