"""CPU ORACLE -- test infrastructure only.

Python face of oracle/kquant_oracle.c, a scalar C restatement of coldpress's numpy k-quant
codec (coldpress/kquant.py) and EF encoder (coldpress/ef.py:46-218).  Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline leg import this module, and only to
check or time against; nothing in perm_b200/ may import it.

Parity pin: tests/golden/ holds outputs of the reference itself (tests/golden/make_golden.py);
tests/test_oracle_golden.py requires this oracle to reproduce them byte for byte.

The function names and signatures mirror the reference so the tests read alike:
    QUANTIZE[t](x, qw) -> uint8 [nrow, n/256*B]        (kquant.py:732)
    DEQUANTIZE[t](raw, n) -> f32 [nrow, n]              (kquant.py:734)
    cholesky_inv_upper(H, damp) -> U f64                (ef.py:46-84)
    ef_encode(x, ttype, qw, H, n_iter, damp, act_order) (ef.py:179-218)
"""
import ctypes
import os
import subprocess
import sys

import numpy as np

F32 = np.float32
_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "_build", "libkqoracle.so")

TYPE_ID = {"Q8_0": 8, "Q2_K": 10, "Q3_K": 11, "Q4_K": 12, "Q5_K": 13, "Q6_K": 14}
BYTES_PER_BLOCK = {"Q2_K": 84, "Q3_K": 110, "Q4_K": 144, "Q5_K": 176, "Q6_K": 210, "Q8_0": 34}
BLOCK_ELEMS = {"Q2_K": 256, "Q3_K": 256, "Q4_K": 256, "Q5_K": 256, "Q6_K": 256, "Q8_0": 32}
# (sub-block width, code lo, code hi, has a min) per type, as in ef.py:87-127.
GRID = {"Q2_K": (16, 0, 3, True), "Q3_K": (16, -4, 3, False), "Q4_K": (32, 0, 15, True),
        "Q5_K": (32, 0, 31, True), "Q6_K": (16, -32, 31, False)}


def build(force=False):
    """Compile kquant_oracle.c with gcc (no FMA contraction: each numpy op rounds once)."""
    src = os.path.join(_HERE, "kquant_oracle.c")
    if (not force and os.path.exists(_LIB_PATH)
            and os.path.getmtime(_LIB_PATH) >= os.path.getmtime(src)):
        return _LIB_PATH
    os.makedirs(os.path.dirname(_LIB_PATH), exist_ok=True)
    cmd = ["gcc", "-O2", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off", "-fno-fast-math",
           "-std=c11", "-Wall", "-o", _LIB_PATH, src, "-lm"]
    subprocess.run(cmd, check=True)
    return _LIB_PATH


_lib = None


def lib():
    global _lib
    if _lib is None:
        path = _LIB_PATH if os.path.exists(_LIB_PATH) else build()
        L = ctypes.CDLL(path)
        P, I64, I = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
        L.kqo_quantize.argtypes = [I, P, I64, I64, P, P, I]
        L.kqo_dequantize.argtypes = [I, P, I64, I64, P, I]
        L.kqo_grid_params.argtypes = [I, P, I64, I64, P, P]
        L.kqo_codes.argtypes = [I, P, I64, I64, P]
        L.kqo_repack.argtypes = [I, P, P, I64, I64]
        L.kqo_ef_sweep.argtypes = [P, I64, I64, P, P, P, P, I, I, I, P, P, I]
        for f in (L.kqo_quantize, L.kqo_dequantize, L.kqo_grid_params, L.kqo_codes,
                  L.kqo_repack, L.kqo_ef_sweep):
            f.restype = I
        _lib = L
    return _lib


def _ptr(a):
    return ctypes.c_void_p(a.ctypes.data) if a is not None else None


def _check(rc, what):
    if rc != 0:
        raise ValueError(f"oracle {what} failed with status {rc}")


def quantize(ttype, x, qw=None, nthreads=0):
    x = np.ascontiguousarray(x, dtype=F32)
    nrow, n = x.shape
    assert n % BLOCK_ELEMS[ttype] == 0
    if qw is not None:
        qw = np.ascontiguousarray(np.broadcast_to(np.asarray(qw, F32), (n,)))
    out = np.zeros((nrow, n // BLOCK_ELEMS[ttype] * BYTES_PER_BLOCK[ttype]), np.uint8)
    _check(lib().kqo_quantize(TYPE_ID[ttype], _ptr(x), nrow, n, _ptr(qw), _ptr(out), nthreads),
           "quantize")
    return out


def dequantize(ttype, raw, n, nthreads=0):
    raw = np.ascontiguousarray(raw, dtype=np.uint8)
    nrow = raw.shape[0]
    out = np.zeros((nrow, n), F32)
    _check(lib().kqo_dequantize(TYPE_ID[ttype], _ptr(raw), nrow, n, _ptr(out), nthreads),
           "dequantize")
    return out


QUANTIZE = {t: (lambda x, qw=None, _t=t: quantize(_t, x, qw)) for t in TYPE_ID}
DEQUANTIZE = {t: (lambda raw, n, _t=t: dequantize(_t, raw, n)) for t in TYPE_ID}


def roundtrip(x, ttype, qw=None):
    return dequantize(ttype, quantize(ttype, x, qw), x.shape[1])


def grid_params(ttype, raw, nrow, n):
    sbw = GRID[ttype][0]
    dl = np.zeros((nrow, n // sbw), F32)
    ml = np.zeros((nrow, n // sbw), F32)
    _check(lib().kqo_grid_params(TYPE_ID[ttype], _ptr(np.ascontiguousarray(raw)), nrow, n,
                                 _ptr(dl), _ptr(ml)), "grid_params")
    return dl, ml


def codes(ttype, raw, nrow, n):
    """Signed integer codes [nrow, n] held by committed container bytes."""
    out = np.zeros((nrow, n), np.int32)
    _check(lib().kqo_codes(TYPE_ID[ttype], _ptr(np.ascontiguousarray(raw)), nrow, n, _ptr(out)),
           "codes")
    return out


def repack(ttype, raw, L, nrow, n):
    b = np.ascontiguousarray(raw).copy()
    L = np.ascontiguousarray(L, dtype=np.int32)
    _check(lib().kqo_repack(TYPE_ID[ttype], _ptr(b), _ptr(L), nrow, n), "repack")
    return b


def cholesky_inv_upper(H, damp=0.01, _max_tries=6):
    """ef.py:46-84: U = chol(inv(H + (damp*mean(diag H) + 1e-8) I)).T in float64, with the
    damping escalated x10 (up to 6 tries) when LAPACK reports a non-PD matrix."""
    n = H.shape[0]
    H = H.astype(np.float64).copy()
    mean_diag = float(np.mean(np.diag(H)))
    base = mean_diag if mean_diag > 0.0 else 1.0
    d = damp
    for _ in range(_max_tries):
        Hd = H.copy()
        Hd[np.diag_indices(n)] += d * base + 1e-8
        try:
            Hinv = np.linalg.inv(Hd)
            Hinv = (Hinv + Hinv.T) / 2
            return np.ascontiguousarray(np.linalg.cholesky(Hinv).T)
        except np.linalg.LinAlgError:
            d *= 10.0
    raise np.linalg.LinAlgError(f"oracle cholesky_inv_upper: not PD after damp {d / 10.0:g}")


def ef_sweep(x, order, U32, dl, ml, ttype, nthreads=0):
    """One EF pass (ef.py:197-216): returns (codes [nrow,n] int32, compensated w [nrow,n])."""
    x = np.ascontiguousarray(x, dtype=F32)
    nrow, n = x.shape
    sbw, lo, hi, has_min = GRID[ttype]
    order = np.ascontiguousarray(order, dtype=np.int64)
    U32 = np.ascontiguousarray(U32, dtype=F32)
    dl = np.ascontiguousarray(dl, dtype=F32)
    mlp = np.ascontiguousarray(ml, dtype=F32) if has_min else None
    L = np.zeros((nrow, n), np.int32)
    wf = np.zeros((nrow, n), F32)
    _check(lib().kqo_ef_sweep(_ptr(x), nrow, n, _ptr(order), _ptr(U32), _ptr(dl), _ptr(mlp),
                              sbw, lo, hi, _ptr(L), _ptr(wf), nthreads), "ef_sweep")
    return L, wf


def ef_encode(x, ttype, qw, H, n_iter=2, damp=0.01, act_order=True, nthreads=0, U=None):
    """ef.py:179-218 restated: returns (raw bytes, recon)."""
    x = np.ascontiguousarray(x, dtype=F32)
    nrow, n = x.shape
    order = np.argsort(-np.diag(H)) if act_order else np.arange(n)
    if U is None:
        Hp = H[np.ix_(order, order)]
        U = cholesky_inv_upper(Hp, damp).astype(F32)
    w_cur = x.copy()
    raw = None
    for _ in range(n_iter):
        raw = quantize(ttype, w_cur, qw, nthreads)
        dl, ml = grid_params(ttype, raw, nrow, n)
        L, w_cur = ef_sweep(x, order, U, dl, ml, ttype, nthreads)
        raw = repack(ttype, raw, L, nrow, n)
    return raw, dequantize(ttype, raw, n)


if __name__ == "__main__":
    print(build(force="--force" in sys.argv))
