"""Generate the golden fixtures that pin the CPU oracle to the reference implementation.

Run in a container where the reference coldpress package is importable:

    python tests/golden/make_golden.py --ref /path/to/reference/source/tree

It imports the reference's own kquant.py and ef.py, feeds them seeded synthetic inputs and
stores inputs and outputs (bytes, reconstructions, the float32 U factor) as .npz files next
to this script.  Inputs are stored, not regenerated, because numpy's random streams and BLAS
kernels are not guaranteed bit-stable across machines.  The tests never import the reference;
they compare the oracle (and, on a GPU, the CUDA path) against these files.
"""
import argparse
import os
import platform
import sys

import numpy as np

F32 = np.float32
HERE = os.path.dirname(os.path.abspath(__file__))
TYPES = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K", "Q8_0"]
K_TYPES = ["Q2_K", "Q3_K", "Q4_K", "Q5_K", "Q6_K"]


def kquant_inputs(rng):
    """Three [8, 1024] weight sets: Student-t(3) tails, cubic heavy tails, and edge cases."""
    t3 = (rng.standard_t(3, size=(8, 1024)) * 0.02).astype(F32)
    cubic = ((rng.standard_normal((8, 1024)) ** 3)
             * rng.uniform(0.2, 3.0, size=(8, 1)).astype(F32)).astype(F32)
    e = (rng.standard_normal((8, 1024)) * 0.02).astype(F32)
    e[0, :256] = 0.0                                   # all-zero superblock
    e[1, :256] = -0.0                                  # all negative-zero superblock
    e[2, :16] = 0.5                                    # constant sub-block
    e[2, 256:512] = 0.25                               # constant superblock
    e[3, :256] = 1e-20                                 # below the 1e-15 group epsilon
    e[4, :32] = np.abs(e[4, :32])                      # non-negative sub-blocks
    e[5, :256] = -np.abs(e[5, :256])                   # non-positive superblock
    e[6, ::7] = 0.0                                    # scattered zeros
    e[7, :256] = np.round(e[7, :256] * 100) / 100      # many exact ties
    e[7, 512:768] = rng.standard_normal(256).astype(F32) * 3e4   # large magnitudes
    e[6, 768:784] = 0.0
    e[6, 770] = 1.0                                    # one-hot sub-block
    return {"t3": t3, "cubic": cubic, "edge": e}


def correlated_hessian(n, T, rng):
    mix = rng.standard_normal((n, n)) / np.sqrt(n) + 1.5 * np.eye(n)
    X = rng.standard_normal((T, n)) @ mix.T
    return X.T @ X


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="source tree of the reference (the directory holding coldpress/)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from coldpress import kquant as kq, ef

    rng = np.random.default_rng(20261201)
    meta = {"numpy": np.__version__, "machine": platform.machine(),
            "processor": platform.processor() or "unknown"}

    # ---- plain k-quant: bytes of every type, imatrix and reference paths, plus decodes
    xs = kquant_inputs(rng)
    qw = rng.lognormal(0.0, 1.0, 1024).astype(F32)
    qw0 = qw.copy()
    qw0[::5] = 0.0                                     # dead imatrix channels
    out = {}
    for name, x in xs.items():
        out[f"x/{name}"] = x
        for qname, q in (("imat", qw), ("imat0", qw0), ("ref", None)):
            for t in TYPES:
                raw = kq.QUANTIZE[t](x, q)
                out[f"raw/{name}/{qname}/{t}"] = raw
                if name == "t3":
                    out[f"deq/{name}/{qname}/{t}"] = kq.DEQUANTIZE[t](raw, x.shape[1])
    out["qw"] = qw
    out["qw0"] = qw0
    np.savez_compressed(os.path.join(HERE, "kquant_golden.npz"), **out,
                        **{f"meta/{k}": np.array(v) for k, v in meta.items()})

    # ---- EF: n = 512, 16 rows per type, one correlated Hessian shared by all types
    n, nrow, T = 512, 16, 4096
    H = correlated_hessian(n, T, rng).astype(F32)     # stored as float32, used as float64
    H64 = H.astype(np.float64)
    qw_ef = (np.diag(H64) / T).astype(F32)
    order = np.argsort(-np.diag(H64))
    U = ef.cholesky_inv_upper(H64[np.ix_(order, order)], 0.01).astype(F32)
    iu = np.triu_indices(n)
    ef_out = {"H": H, "qw": qw_ef, "order": order.astype(np.int64), "U_upper": U[iu]}
    for t in K_TYPES:
        W = (rng.standard_normal((nrow, n)) ** 3).astype(F32)
        W[:, rng.choice(n, 5, replace=False)] *= 8.0   # outlier input channels
        ef_out[f"W/{t}"] = W
        for qname, q in (("imat", qw_ef), ("ref", None)):
            raw, recon = ef.ef_encode(W, t, q, H64, n_iter=2, act_order=True)
            ef_out[f"raw/{qname}/{t}"] = raw
            ef_out[f"recon/{qname}/{t}"] = recon
        raw1, _ = ef.ef_encode(W, t, qw_ef, H64, n_iter=1, act_order=True)
        ef_out[f"raw1/imat/{t}"] = raw1
        raws, _ = ef.ef_encode(W, t, qw_ef, H64, n_iter=2, act_order=False)
        ef_out[f"raw_storage/imat/{t}"] = raws
    np.savez_compressed(os.path.join(HERE, "ef_golden.npz"), **ef_out)

    # ---- factorization with escalation: one clearly negative eigenvalue (n = 128)
    m = 128
    Q, _ = np.linalg.qr(rng.standard_normal((m, m)))
    eig = np.linspace(1.0, 100.0, m)
    eig[0] = -2.0
    Hbad = (Q * eig) @ Q.T
    Hbad = (Hbad + Hbad.T) / 2
    Ubad = ef.cholesky_inv_upper(Hbad, damp=0.01)
    Mpd = rng.standard_normal((m, m))
    Hpd = Mpd @ Mpd.T + m * np.eye(m)
    Upd = ef.cholesky_inv_upper(Hpd, damp=0.01)
    np.savez_compressed(os.path.join(HERE, "factor_golden.npz"), H_bad=Hbad, U_bad=Ubad,
                        H_pd=Hpd, U_pd=Upd)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))


if __name__ == "__main__":
    main()
