"""Generate the config-sized golden digests that pin the CUDA path to the reference itself.

Run in a container where the reference's source tree is available:

    python tests/golden/make_golden_config.py --ref /path/to/reference/source/tree

It regenerates BASELINE config[1] (plain imatrix-weighted k-quant of a 4096 x 4096 Student-t
tensor, all five k-quant types on the imatrix and the reference path) and config[0] (EF
Q2_K of a 3072 x 1024 tensor with outlier columns) from fixed seeds, runs the reference's
own kquant.QUANTIZE and ef.ef_encode on them, and stores in config_golden.npz:
  * the SHA-256 of each generated input, so a test can prove it rebuilt the same inputs;
  * the SHA-256 of each config[1] output (5 types x 2 paths; 16 MiB of inputs do not fit a
    fixture, the digests do);
  * the config[0] EF output bytes themselves (1 MiB).
The inputs are rebuilt by tests/golden/config_inputs.py, which the tests import too.
"""
import argparse
import hashlib
import os
import sys
import time

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import config_inputs as ci  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="source tree of the reference (the directory holding coldpress/)")
    args = ap.parse_args()
    sys.path.insert(0, args.ref)
    from coldpress import ef, kquant as kq
    out = {}
    W1, qw1 = ci.config1()
    out["c1_W_sha"] = np.array(ci.sha(W1))
    out["c1_qw_sha"] = np.array(ci.sha(qw1))
    for tt in ci.K_TYPES:
        for path, qw in (("imat", qw1), ("ref", None)):
            t0 = time.time()
            raw = kq.QUANTIZE[tt](W1, qw)
            out[f"c1_{tt}_{path}_sha"] = np.array(ci.sha(raw))
            out[f"c1_{tt}_{path}_shape"] = np.array(raw.shape)
            print(f"config1 {tt} {path}: {time.time() - t0:.1f}s", flush=True)
    W0, H0, qw0 = ci.config0()
    out["c0_W_sha"] = np.array(ci.sha(W0))
    out["c0_H_sha"] = np.array(ci.sha(H0))
    t0 = time.time()
    raw0, _ = ef.ef_encode(W0, "Q2_K", qw0, H0, n_iter=2, damp=0.01, act_order=True)
    print(f"config0 EF: {time.time() - t0:.1f}s", flush=True)
    out["c0_raw"] = np.ascontiguousarray(raw0, np.uint8)
    np.savez_compressed(os.path.join(HERE, "config_golden.npz"), **out)


if __name__ == "__main__":
    main()
