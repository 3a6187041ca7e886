"""Small, fixed micro-cases of the encoder's kernels, for timing and for profiler captures
(`ncu ... python bench_cases.py <case>`).  Each case holds at most a few hundred MB
on the device (llama_layers: about 30 GB) and runs its kernels a few times.

    sweep    24 Q2_K tensors 1024 x 1024 plus 8 Q3_K tensors 1024 x 3072, grouped EF sweep
    sweep_wide    40 Q2_K tensors 4096 x 1024, the ordinary (unsplit) sweep form
    sweep_layers  eight Qwen3-0.6B-shaped layers (56 tensors), grouped EF sweep
    sweep_model   all 28 layers' EF tensors (196 tensors), the whole-model sweep launch
    fit      Q2_K imatrix fit of a 4096 x 4096 tensor
    factor   batched FP64 factorisation of 16 Hessians n = 1024 and 4 of n = 3072
    factor_model  the whole 0.6B model's 112 factorisations
    factor_rank8  one rank's share of an 8-GPU plan's factorisations (latency-bound)
    llama_layers  four Llama-3-8B-shaped layers streamed in two batches (config[4] pipeline)
    xtx      X^T X of 32768 bf16 tokens at d = 1024, 2048, 3072 (tcgen05 kernel)
    xtx_f32  the same with float32 tokens (hi/lo bf16 split, four products)
"""
import os
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)


def _hess(torch, n, seed, T=4096):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    X = torch.randn(T, n, device="cuda", dtype=torch.float64, generator=g)
    X *= torch.exp(torch.randn(n, device="cuda", dtype=torch.float64, generator=g))
    return X.T @ X / T


def _sweep_case(torch, reps, shapes):
    from perm_b200 import _native as nat
    from perm_b200.encoder import Encoder, Job
    hs, jobs = {}, []
    for i, (nrow, n, tt, hk) in enumerate(shapes):
        if hk not in hs:
            hs[hk] = _hess(torch, n, len(hs) + n)
        x = torch.randn(nrow, n, device="cuda") * 0.02
        jobs.append(Job(f"t{i}", tt, "EF", x, torch.diagonal(hs[hk]).float().contiguous(), hk))
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
    upd = sum(2 * r * n * (n - 1) / 2 for r, n, _, _ in shapes)
    ms = p["sweep"][0] / reps
    return ms, upd


def case_sweep(torch, reps):
    """24 Q2_K tensors 1024 x 1024 + 8 Q3_K tensors 1024 x 3072 (256 CTAs: under one wave)."""
    shapes = [(1024, 1024, "Q2_K", "h1024")] * 24 + [(1024, 3072, "Q3_K", "h3072")] * 8
    ms, upd = _sweep_case(torch, reps, shapes)
    return f"sweep: {ms:.3f} ms per 2-round encode, {upd / ms / 1e9:.2f} T ordered updates/s"


def case_sweep_wide(torch, reps):
    """40 Q2_K tensors 4096 x 1024 over 8 Hessians (1280 CTAs: enough for the ordinary sweep
    form, which launches of fewer than 8 x 148 CTAs do not use), about 3 GB on the device."""
    shapes = [(4096, 1024, "Q2_K", f"h{i % 8}") for i in range(40)]
    ms, upd = _sweep_case(torch, reps, shapes)
    return (f"sweep_wide: {ms:.3f} ms per 2-round encode, {upd / ms / 1e9:.2f} T ordered updates/s, "
            f"{2 * upd / ms / 1e9:.2f} T fp32 lane-ops/s")


def case_sweep_model(torch, reps):
    """All 28 Qwen3-0.6B-shaped layers' EF tensors (196 tensors, 2688 CTAs), each layer with its
    own four Hessians (112 factors, as in the whole-model encode): the whole-model sweep."""
    shapes = []
    for l in range(28):
        shapes += [(2048, 1024, "Q2_K", f"qkv{l}"), (1024, 1024, "Q2_K", f"qkv{l}"), (1024, 1024, "Q2_K", f"qkv{l}"),
                   (1024, 2048, "Q2_K", f"o{l}"), (3072, 1024, "Q2_K", f"gu{l}"), (3072, 1024, "Q2_K", f"gu{l}"),
                   (1024, 3072, "Q3_K", f"d{l}")]
    shapes.sort(key=lambda s: -s[1])
    ms, upd = _sweep_case(torch, reps, shapes)
    return (f"sweep_model: {ms:.3f} ms per 2-round encode, {upd / ms / 1e9:.2f} T ordered updates/s, "
            f"{2 * upd / ms / 1e9:.2f} T fp32 lane-ops/s")


def case_sweep_layers(torch, reps):
    """Eight Qwen3-0.6B-shaped layers (q, k, v, o, gate, up, down; Q2_K/Q3_K mixture shapes),
    each layer with its own four Hessians: 768 CTAs, the whole-model sweep's mix of n."""
    shapes = []
    for l in range(8):
        shapes += [(2048, 1024, "Q2_K", f"qkv{l}"), (1024, 1024, "Q2_K", f"qkv{l}"), (1024, 1024, "Q2_K", f"qkv{l}"),
                   (1024, 2048, "Q2_K", f"o{l}"), (3072, 1024, "Q2_K", f"gu{l}"), (3072, 1024, "Q2_K", f"gu{l}"),
                   (1024, 3072, "Q3_K", f"d{l}")]
    shapes.sort(key=lambda s: -s[1])
    ms, upd = _sweep_case(torch, reps, shapes)
    return (f"sweep_layers: {ms:.3f} ms per 2-round encode, {upd / ms / 1e9:.2f} T ordered updates/s, "
            f"{2 * upd / ms / 1e9:.2f} T fp32 lane-ops/s")


def case_fit(torch, reps):
    from perm_b200 import kquant as kq
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
    from perm_b200.encoder import Encoder
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
    """Flops the tensor cores execute: 256 x 256 pair tiles on or below the diagonal."""
    nT = -(-d // 256)
    return 2.0 * (nT * (nT + 1) // 2) * 256 * 256 * T


def case_factor_model(torch, reps):
    """The whole Qwen3-0.6B-shaped model's 112 factorisations (56 at n = 1024, 28 at 2048,
    28 at 3072) through Encoder.factor, wall time with a device sync."""
    from perm_b200.encoder import Encoder
    base = {1024: _hess(torch, 1024, 1), 2048: _hess(torch, 2048, 2), 3072: _hess(torch, 3072, 3)}
    hs = {}
    for l in range(28):
        for k, n in (("qkv", 1024), ("o", 2048), ("gu", 1024), ("d", 3072)):
            hs[f"{k}{l}"] = base[n] * (1.0 + 0.01 * l)
    ds = {k: torch.diagonal(v).cpu().numpy() for k, v in hs.items()}
    enc = Encoder()
    enc.factor(hs, ds)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        enc.factor(hs, ds)
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t) / reps
    fl = (2.0 / 3.0) * 28 * (2 * 1024 ** 3 + 2048 ** 3 + 3072 ** 3)
    return f"factor_model 112 Hessians: {dt * 1e3:.2f} ms, {fl / dt / 1e12:.2f} FP64 TFLOP/s"


def case_factor_rank8(torch, reps):
    """About one eighth of the 0.6B model's factorisations (3 at n = 3072, 4 at 2048, 7 at
    1024): what one rank of an 8-GPU encode runs, bound by the length of the n = 3072 chain."""
    from perm_b200.encoder import Encoder
    hs = {}
    for i in range(3):
        hs[f"d{i}"] = _hess(torch, 3072, 30 + i)
    for i in range(4):
        hs[f"o{i}"] = _hess(torch, 2048, 20 + i)
    for i in range(7):
        hs[f"q{i}"] = _hess(torch, 1024, 10 + i)
    ds = {k: torch.diagonal(v).cpu().numpy() for k, v in hs.items()}
    enc = Encoder()
    enc.factor(hs, ds)
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        enc.factor(hs, ds)
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t) / reps
    fl = (2.0 / 3.0) * (3 * 3072 ** 3 + 4 * 2048 ** 3 + 7 * 1024 ** 3)
    return f"factor_rank8 3x3072 + 4x2048 + 7x1024: {dt * 1e3:.2f} ms, {fl / dt / 1e12:.2f} FP64 TFLOP/s"


def case_llama_layers(torch, reps):
    """Four Llama-3-8B-shaped layers (q/k/v/o, gate/up 14336 x 4096, down 4096 x 14336; the
    Q4_K_M-style mixture) streamed through Encoder.run_stream in two batches of two layers,
    Hessians resident in storage form (from 8192 synthetic tokens) and decoded per batch: the
    config[4] pipeline at a size a profiler capture can hold (about 25 GB)."""
    from perm_b200 import model, stream as stm
    from perm_b200.encoder import Encoder, Job
    cfg = dict(model.MODELS["llama3-8b"], n_layers=4)
    specs = [sp for sp in model.tensor_specs(cfg, "q4_k_m_style") if sp.name.startswith("blk.")]
    dims = model.hessian_dims(specs)
    stored = {}
    for k, d in dims.items():
        stored[k] = stm.store_hessian(torch, model.synth_hessian(torch, d, k, 0, "cuda", tokens=8192))
    jobs = []
    for sp in specs:
        x = model.synth_weights(torch, sp, 0, "cuda")
        qw = torch.from_numpy(stored[sp.hkey].diag_host.astype(np.float32)).cuda()
        jobs.append(Job(sp.name, sp.ttype, "EF", x, qw, sp.hkey))
    per_layer = sum(j.params for j in jobs) / 4
    plan = stm.plan(jobs, dims, 2 * per_layer * stm.ef_bytes_per_param() + 2 * (stm.hessian_bytes(14336) +
                                                                               3 * stm.hessian_bytes(4096)))
    enc = Encoder()
    dec = torch.cuda.Stream(priority=-1)
    enc.run_stream(stm.batches(torch, plan, stored, None, dec))
    torch.cuda.synchronize()
    t = time.perf_counter()
    for _ in range(reps):
        enc.run_stream(stm.batches(torch, plan, stored, None, dec))
    torch.cuda.synchronize()
    dt = (time.perf_counter() - t) / reps
    params = sum(j.params for j in jobs)
    return f"llama_layers 4 layers, {len(plan)} batches: {dt * 1e3:.1f} ms, {params / dt / 1e6:.0f} Mparams/s"


def case_xtx(torch, reps, dtype="bf16"):
    from perm_b200 import hessians
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


CASES = {"sweep": case_sweep, "sweep_wide": case_sweep_wide, "sweep_layers": case_sweep_layers, "sweep_model": case_sweep_model, "fit": case_fit, "factor": case_factor, "factor_model": case_factor_model, "factor_rank8": case_factor_rank8, "llama_layers": case_llama_layers, "xtx": case_xtx, "xtx_f32": case_xtx_f32}


def main(argv):
    import torch
    reps = 3
    if "--reps" in argv:
        i = argv.index("--reps")
        reps = int(argv[i + 1])
        argv = argv[:i] + argv[i + 2:]
    names = argv or list(CASES)
    for n in names:
        print(CASES[n](torch, reps), flush=True)


if __name__ == "__main__":
    main(sys.argv[1:])
