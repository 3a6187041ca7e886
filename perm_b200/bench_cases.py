"""Small, fixed micro-cases of the encoder's kernels, for timing and for profiler captures
(`ncu ... python -m perm_b200.bench_cases <case>`).  Each case holds at most a few hundred MB
on the device and runs its kernels a few times.

    sweep    24 Q2_K tensors 1024 x 1024 plus 8 Q3_K tensors 1024 x 3072, grouped EF sweep
    fit      Q2_K imatrix fit of a 4096 x 4096 tensor
    factor   batched FP64 factorisation of 16 Hessians n = 1024 and 4 of n = 3072
    xtx      X^T X of 32768 bf16 tokens at d = 1024, 2048, 3072 (tcgen05 kernel)
    xtx_f32  the same with float32 tokens (hi/lo bf16 split, four products)
"""
import sys
import time

import numpy as np


def _hess(torch, n, seed, T=4096):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    X = torch.randn(T, n, device="cuda", dtype=torch.float64, generator=g)
    X *= torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
    return X.T @ X / T


def case_sweep(torch, reps):
    from . import _native as nat
    from .encoder import Encoder, Job
    shapes = [(1024, 1024, "Q2_K")] * 24 + [(1024, 3072, "Q3_K")] * 8
    hs, jobs = {}, []
    for i, (nrow, n, tt) in enumerate(shapes):
        k = f"h{n}"
        if k not in hs:
            hs[k] = _hess(torch, n, n)
        x = torch.randn(nrow, n, device="cuda") * 0.02
        jobs.append(Job(f"t{i}", tt, "EF", x, torch.diagonal(hs[k]).float().contiguous(), k))
    enc = Encoder()
    f = enc.factor(hs)
    enc.encode(jobs, f, stats=False)
    torch.cuda.synchronize()
    nat.profile_enable(True)
    for _ in range(reps):
        enc.encode(jobs, f, stats=False)
    torch.cuda.synchronize()
    nat.profile_enable(False)
    p = nat.profile_collect()
    upd = sum(2 * r * n * (n - 1) / 2 for r, n, _ in shapes)
    ms = p["sweep"][0] / reps
    return f"sweep: {ms:.3f} ms per 2-round encode, {upd / ms / 1e9:.2f} T ordered updates/s"


def case_fit(torch, reps):
    from . import kquant as kq
    x = torch.randn(4096, 4096, device="cuda") * 0.02
    qw = torch.exp(torch.randn(4096, device="cuda"))
    out = kq.quantize_dev("Q2_K", x, qw)
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(reps):
        kq.quantize_dev("Q2_K", x, qw, out=out)
    e.record()
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / reps
    return f"fit Q2_K imatrix 4096x4096: {ms:.3f} ms, {x.numel() / ms / 1e3:.1f} Mparam/s"


def case_factor(torch, reps):
    from .encoder import Encoder
    hs = {f"a{i}": _hess(torch, 1024, i) for i in range(16)}
    hs.update({f"b{i}": _hess(torch, 3072, 100 + i) for i in range(4)})
    ds = {k: torch.diagonal(v).cpu().numpy() for k, v in hs.items()}
    enc = Encoder()
    enc.factor(hs, ds)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        enc.factor(hs, ds)
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t) / reps
    fl = (2.0 / 3.0) * (16 * 1024 ** 3 + 4 * 3072 ** 3)
    return f"factor 16x1024 + 4x3072: {dt * 1e3:.2f} ms, {fl / dt / 1e12:.2f} FP64 TFLOP/s"


def _xtx_tile_flops(T, d):
    """Flops the tensor cores execute: 128 x 256 tiles on or below the diagonal."""
    nt = -(-d // 128)
    tiles = sum(ti // 2 + 1 for ti in range(nt))
    return 2.0 * tiles * 128 * 256 * T


def case_xtx(torch, reps, dtype="bf16"):
    from . import hessians
    out = []
    T = 32768
    for d in (1024, 2048, 3072):
        g = torch.Generator(device="cuda")
        g.manual_seed(d)
        X = torch.randn(T, d, device="cuda", generator=g) * torch.exp(torch.randn(d, device="cuda", generator=g))
        X = X.to(torch.bfloat16) if dtype == "bf16" else X
        H = torch.zeros(d, d, device="cuda")
        hessians.xtx_accumulate(X, H)
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        for _ in range(reps):
            hessians.xtx_accumulate(X, H)
        e.record()
        torch.cuda.synchronize()
        hessians.xtx_status()
        ms = s.elapsed_time(e) / reps
        mult = 4 if dtype == "f32" else 1
        out.append(f"xtx {dtype} T={T} d={d}: {ms:.3f} ms, {2 * T * d * d / ms / 1e9:.1f} TFLOP/s (x^T x), "
                   f"{mult * _xtx_tile_flops(T, d) / ms / 1e9:.1f} TFLOP/s on the tensor cores")
    return "; ".join(out)


def case_xtx_f32(torch, reps):
    return case_xtx(torch, reps, "f32")


CASES = {"sweep": case_sweep, "fit": case_fit, "factor": case_factor, "xtx": case_xtx, "xtx_f32": case_xtx_f32}


def main(argv):
    import torch
    names = argv or list(CASES)
    reps = 3
    for n in names:
        print(CASES[n](torch, reps), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
