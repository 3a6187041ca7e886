#!/usr/bin/env python3
"""Benchmark: whole-model error-feedback k-quant encode (coldpress `encode_gguf`'s hot path).

Workload: a Qwen3-0.6B-shaped model (28 layers, hidden 1024, 16 q / 8 kv
heads x 128, ffn 3072, vocab 151936; 198 tensors, 751.6 M parameters) with random-init
N(0, 0.02) weights and synthetic Hessians H = X^T X / T (X = N(0,1) x per-channel
log-normal(0,1) scales, bf16 activations), encoded with error feedback (n_iter 2, damp 0.01,
act order) into the Q2_K mixture (Q2_K q/k/gate/up/token_embd, Q3_K v/o/down, Q6_K output);
token_embd gets the attn0-diagonal weighted RTN, every tensor the stock-baseline statistics.

One step = the whole model: factorise every distinct Hessian, encode every tensor, reduce the
statistics, and (N > 1) gather all packed bytes to rank 0 over NCCL.  Tensors are sharded by
(tensor, row range) units with a cost-balanced greedy assignment; no data moves during
compute.  Inputs are resident in HBM before the timed region (they are larger than L2).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

`--impl reference` times the reference algorithm on the host cores through the CPU oracle
(the reference is pure Python/numpy and cannot run on the GPU box): each step encodes one
full transformer layer (7 tensors, 25.2 M parameters) with all host threads.
"""
import argparse
import json
import os
import subprocess
import sys
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "EF-encoded Mparams/s (Q2_K)"
UNIT = "Mparams/s"
L2_BYTES = 126 * 2 ** 20


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--model", default="qwen3-0.6b")
    ap.add_argument("--mixture", default="q2_k_mix")
    ap.add_argument("--hessian-tokens", type=int, default=262144)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ----------------------------------------------------------------------------- clocks

class ClockSampler:
    """nvidia-smi clocks and throttle reasons sampled every 200 ms during the timed region."""
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.proc = None
        self.path = os.path.join("/tmp", f"bench_clocks_{os.getpid()}.csv")

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.QUERY}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        sm, smax, reasons = [], [], set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in open(self.path):
            f = [c.strip() for c in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                smax.append(float(f[2]))
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        try:
            os.unlink(self.path)
        except OSError:
            pass
        if not sm:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        return {"sm_mhz": float(np.median(sm)), "sm_max_mhz": max(smax), "samples": len(sm),
                "reasons": sorted(reasons)}


# ----------------------------------------------------------------------------- CPU (oracle) arm

def layer_sample(seed, layer=0):
    """One Qwen3-0.6B-shaped layer on the host: [(name, W f32, qw, H f64, type)]."""
    from perm_b200 import model
    cfg = model.MODELS["qwen3-0.6b"]
    specs = [s for s in model.tensor_specs(cfg, "q2_k_mix") if s.name.startswith(f"blk.{layer}.")]
    rng = np.random.default_rng(seed)
    hs = {}
    out = []
    for s in specs:
        if s.hkey not in hs:
            T = 8192
            X = rng.standard_normal((T, s.n)).astype(np.float32) * rng.lognormal(0, 1, s.n).astype(np.float32)
            hs[s.hkey] = (X.T.astype(np.float64) @ X.astype(np.float64)) / T
        H = hs[s.hkey]
        W = (rng.standard_normal((s.nrow, s.n)) * 0.02).astype(np.float32)
        out.append((s.name, W, np.diag(H).astype(np.float32), H, s.ttype))
    return out


def cpu_encode_layer(sample, nthreads):
    from oracle import oracle as orc
    n_params = 0
    for name, W, qw, H, tt in sample:
        orc.ef_encode(W, tt, qw, H, n_iter=2, act_order=True, nthreads=nthreads)
        orc.roundtrip(W, tt, qw)  # encode_gguf's stock baseline (ef.py:298)
        n_params += W.size
    return n_params


def cpu_threads():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_cpu_baseline(seed, reps=1):
    from oracle import oracle as orc
    orc.build()
    sample = layer_sample(seed)
    nt = cpu_threads()
    t0 = time.perf_counter()
    n = 0
    for _ in range(reps):
        n += cpu_encode_layer(sample, nt)
    dt = time.perf_counter() - t0
    return {"value": n / dt / 1e6, "unit": UNIT, "cores": nt, "kind": "port",
            "sample": "layer 0 of the Qwen3-0.6B-shaped model (7 tensors, 25.2 M params): EF n_iter 2 "
                      "(numpy LAPACK factor + C oracle fits/sweeps) plus the stock-baseline roundtrip, "
                      "H from 8192 tokens", "seconds": dt}


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    from oracle import oracle as orc
    orc.build()
    sample = layer_sample(args.seed)
    nt = cpu_threads()
    for _ in range(args.warmup):
        cpu_encode_layer(sample, nt)
    t0 = time.perf_counter()
    n = 0
    for _ in range(args.steps):
        n += cpu_encode_layer(sample, nt)
    dt = time.perf_counter() - t0
    value = n / dt / 1e6
    line = {"metric": METRIC, "value": value, "unit": UNIT, "impl": "reference", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": dt / args.steps * 1e3,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic",
            "config": {"workload": "reference CPU encoder (oracle port), one Qwen3-0.6B-shaped layer per step",
                       "mixture": args.mixture, "n_iter": 2, "act_order": True, "damp": 0.01},
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": nt, "kind": "port",
                             "sample": "layer 0 of the Qwen3-0.6B-shaped model per step (7 tensors, 25.2 M params)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm

class Workload:
    """Inputs of this rank's units, resident on the device."""

    def __init__(self, torch, args, rank, world):
        from perm_b200 import model, shard
        self.torch = torch
        cfg = model.MODELS[args.model]
        self.specs = model.tensor_specs(cfg, args.mixture)
        self.spec_by_name = {s.name: s for s in self.specs}
        metas = [shard.UnitMeta(s.name, s.ttype, s.mode, s.nrow, s.n, s.hkey, s.mode != "wRTN(attn0-diag)")
                 for s in self.specs]
        self.plan = shard.make_plan(metas, world)
        self.units = self.plan.units[rank]
        self.total_params = sum(s.params for s in self.specs)
        dims = model.hessian_dims(self.specs)
        need = set()
        for u in self.units:
            sp = self.spec_by_name[u.name]
            need.add(sp.hkey)
        self.hess, self.diags = {}, {}
        for k in sorted(need):
            H = model.synth_hessian(torch, dims[k], k, args.seed, "cuda", tokens=args.hessian_tokens)
            self.hess[k] = H
            self.diags[k] = torch.diagonal(H).cpu().numpy()
        self.ef_keys = sorted({self.spec_by_name[u.name].hkey for u in self.units
                               if self.spec_by_name[u.name].mode == "EF"})
        # the rank's weights are views into one flat float32 buffer (e2e moves them with one
        # copy and one conversion)
        total = sum((u.r1 - u.r0) * self.spec_by_name[u.name].n for u in self.units)
        self.x_flat = torch.empty(max(1, total), dtype=torch.float32, device="cuda")
        self.x = {}
        full_cache = {}
        off = 0
        for u in self.units:
            sp = self.spec_by_name[u.name]
            if sp.name not in full_cache:
                full_cache = {sp.name: model.synth_weights(torch, sp, args.seed, "cuda")}
            cnt = (u.r1 - u.r0) * sp.n
            v = self.x_flat[off:off + cnt].view(u.r1 - u.r0, sp.n)
            v.copy_(full_cache[sp.name][u.r0:u.r1])
            self.x[self.uid(u)] = v
            off += cnt
        del full_cache
        self.qw = {k: torch.from_numpy(self.diags[k].astype(np.float32)).cuda() for k in self.diags}

    @staticmethod
    def uid(u):
        return f"{u.name}[{u.r0}:{u.r1}]"

    def jobs(self):
        from perm_b200.encoder import Job
        out = []
        for u in self.units:
            sp = self.spec_by_name[u.name]
            x = self.x[self.uid(u)]
            if sp.mode == "EF":
                out.append(Job(self.uid(u), sp.ttype, "EF", x, self.qw[sp.hkey], sp.hkey))
            else:  # token_embd: no imatrix entry; fit weights diag(H_blk0_attn_q)/n0
                out.append(Job(self.uid(u), sp.ttype, sp.mode, x, None, None, fit_w=self.qw[sp.hkey]))
        return out

    def out_bytes(self):
        from perm_b200 import kquant as kq
        sizes = []
        for u in self.units:
            sp = self.spec_by_name[u.name]
            sizes.append((u.r1 - u.r0) * kq.row_bytes(sp.ttype, sp.n))
        return sizes

    def algorithmic(self, n_iter=2):
        """Per-step algorithmic work of this rank per kernel class."""
        from perm_b200 import kquant as kq
        fit_bytes = fit_evals = sweep_updates = sweep_bytes = 0.0
        factor_flops = sum((2.0 / 3.0) * float(self.hess[k].shape[0]) ** 3 for k in self.ef_keys)
        from perm_b200.shard import FIT_PASSES
        for u in self.units:
            sp = self.spec_by_name[u.name]
            rows = u.r1 - u.r0
            nfit = n_iter if sp.mode == "EF" else 2
            imat = sp.mode == "EF" or sp.mode == "wRTN(attn0-diag)"
            fit_bytes += nfit * (rows * sp.n * 4 + sp.n * 4 + rows * kq.row_bytes(sp.ttype, sp.n))
            fit_evals += nfit * rows * sp.n * FIT_PASSES[(sp.ttype, imat)]
            if sp.mode == "EF":
                sweep_updates += n_iter * rows * sp.n * (sp.n - 1) / 2.0
                sweep_bytes += n_iter * (rows * sp.n * (4 + 1 + 4)) + n_iter * sp.n * sp.n * 2.0
        return {"fit_bytes": fit_bytes, "fit_evals": fit_evals, "sweep_updates": sweep_updates,
                "sweep_bytes": sweep_bytes, "factor_flops": factor_flops}


def gpu_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from perm_b200 import _native as nat
    from perm_b200.encoder import Encoder
    from perm_b200.shard import gather_to_rank0

    torch.cuda.set_device(local_rank)
    nat.lib()
    wl = Workload(torch, args, rank, world)
    jobs = wl.jobs()
    sizes = wl.out_bytes()
    my_bytes = int(sum(sizes))
    flat = torch.empty(max(1, my_bytes), dtype=torch.uint8, device="cuda")
    outputs, off = {}, 0
    for u, sz, j in zip(wl.units, sizes, jobs):
        rows = u.r1 - u.r0
        outputs[j.name] = flat[off:off + sz].view(rows, sz // rows)
        off += sz
    all_sizes = [0] * world
    if world > 1:
        t = torch.tensor([my_bytes], dtype=torch.int64, device="cuda")
        g = [torch.zeros(1, dtype=torch.int64, device="cuda") for _ in range(world)]
        dist.all_gather(g, t)
        all_sizes = [int(v.item()) for v in g]
    else:
        all_sizes = [my_bytes]
    enc = Encoder(n_iter=2, damp=0.01, act_order=True)

    def step():
        _, st = enc.run(jobs, {k: wl.hess[k] for k in wl.ef_keys}, {k: wl.diags[k] for k in wl.ef_keys},
                        stats=True, outputs=outputs)
        if world > 1:
            gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
        return st

    if world > 1:
        dist.barrier()
    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    time.sleep(0.3)
    launches0 = nat.lib().cp_launch_count()
    nat.profile_enable(True)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t_start.record()
    for _ in range(args.steps):
        st = step()
    t_end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    nat.profile_enable(False)
    launches = (nat.lib().cp_launch_count() - launches0) // max(1, args.steps)
    prof = nat.profile_collect()
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = wl.total_params / (ms / 1e3) / 1e6

    # dominant kernel class and its roofline (this rank's algorithmic work / its event time)
    from perm_b200 import _native as _n  # noqa: F401
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    peak_src = "measured" if "hbm_gbs" in peaks else "fallback"
    alg = wl.algorithmic()
    per_step = {c: (prof[c][0] / args.steps, prof[c][1] / args.steps) for c in prof}
    # The sweep is the dominant kernel by serialised device time (ncu launch list of this
    # command).  Class event times cannot pick it: the factor chains run on side streams next
    # to the fits, so their event spans include the overlap.
    dom = "sweep" if per_step["sweep"][1] > 0 else max(("fit", "factor"), key=lambda c: per_step[c][0])
    sm_mhz = clk.get("sm_mhz") or 1965.0
    alu_peak = 148 * 128 * sm_mhz * 1e6 / 1e12  # T fp32 lane-ops/s (FADD/FMUL/FFMA each one lane-op)
    kms = per_step[dom][0]
    nl = max(1.0, per_step[dom][1])
    if dom == "sweep":
        gbs = alg["sweep_bytes"] / (kms / 1e3) / 1e9
        alu = {"achieved": 2.0 * alg["sweep_updates"] / (kms / 1e3) / 1e12, "peak": alu_peak,
               "unit": "T fp32 lane-ops/s", "work": "2 unfused ops per ordered update"}
    elif dom == "fit":
        gbs = alg["fit_bytes"] / (kms / 1e3) / 1e9
        alu = {"achieved": 20.0 * alg["fit_evals"] / (kms / 1e3) / 1e12, "peak": alu_peak,
               "unit": "T fp32 lane-ops/s", "work": "~20 ops per candidate-element evaluation"}
    else:
        gbs = None
        alu = {"achieved": alg["factor_flops"] / (kms / 1e3) / 1e12, "peak": 37.0,
               "unit": "FP64 TFLOP/s (nominal peak)", "work": "(2/3) n^3 per factorisation"}
    if alu.get("peak"):
        alu["frac"] = alu["achieved"] / alu["peak"]
    traffic = None
    if dom == "sweep":
        # DRAM bytes of one sweep launch: ncu (dram__bytes_read.sum + dram__bytes_write.sum) of
        # the second step's first sweep launch of this default workload on one B200 measured
        # 36.77 GB (31.37 read + 5.40 written) for 425.1 G ordered updates, 0.08649 bytes per
        # update; per launch of this rank = that rate x this rank's updates per round
        traffic = 0.08649 * alg["sweep_updates"] / max(1.0, nl)
    roofline = {"kernel": {"fit": "kquant fit+pack", "sweep": "ef_sweep", "factor": "fp64 factor"}[dom],
                "bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s",
                "frac": (gbs / hbm) if gbs is not None else None, "traffic": traffic,
                "traffic_unit": "bytes per launch (ncu, scaled by this rank's updates)",
                "peak_source": f"{peak_src} hbm_gbs", "launches_per_step": nl,
                "ms_per_step": kms, "alu": alu,
                "classes_ms_per_step": {c: round(per_step[c][0], 4) for c in per_step}}

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(torch, dist, args, wl, enc, jobs, outputs, flat, my_bytes, all_sizes, rank, world)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline(args.seed)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "whole_model_seconds": ms / 1e3,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (random-init N(0,0.02) weights, synthetic X^T X Hessians)",
                "config": {"workload": f"{args.model}-shaped whole-model EF encode, {args.mixture} "
                                       f"({len(wl.specs)} tensors, {wl.total_params / 1e6:.1f} M params)",
                           "mixture": args.mixture, "n_iter": 2, "damp": 0.01, "act_order": True,
                           "hessian_tokens": args.hessian_tokens,
                           "l2": "inputs (3 GB weights + float64 Hessians) are larger than L2; no flush",
                           "parallelism": f"tensor/row-range shards over {world} GPU(s), NCCL gather of packed bytes"},
                "gpu_launches": int(launches), "roofline": roofline, "clocks": clk, "e2e": e2e,
                "cpu_baseline": cpu, "stats_median_rel_err_vs_stock": float(np.median(
                    [v["rel_err_vs_stock"] for v in st.values()])) if st else None}
        print(json.dumps(line), flush=True)
    return 0


def measure_e2e(torch, dist, args, wl, enc, jobs, outputs, flat, my_bytes, all_sizes, rank, world):
    """Same encode through host buffers: weights as float16 (the GGUF source dtype) and Hessians
    in the reference's storage form (float16 / hscale + exact float32 diagonal) copied from
    pinned memory every step, packed bytes copied back to pinned memory."""
    from perm_b200 import _native as nat
    from perm_b200.shard import gather_to_rank0
    # weights: one pinned float16 image of the rank's flat float32 buffer
    host_w = wl.x_flat.to(torch.float16).cpu().pin_memory()
    dev_w16 = torch.empty_like(host_w, device="cuda")
    # Hessians in stored form, one pinned float16 image per size, diagonals in one buffer
    keys = wl.ef_keys + [k for k in wl.hess if k not in wl.ef_keys]
    by_size = {}
    for k in keys:
        by_size.setdefault(int(wl.hess[k].shape[0]), []).append(k)
    host_h16, dev_h16, hscale, h_off = {}, {}, {}, {}
    diag_parts, d_off, dn = [], {}, 0
    for n, ks in by_size.items():
        parts, off = [], 0
        for k in ks:
            H = wl.hess[k].float()
            amax = float(H.abs().max())
            hscale[k] = amax / 32768.0 if amax > 32768.0 else 1.0
            parts.append((H / hscale[k]).to(torch.float16).reshape(-1))
            h_off[k] = off
            off += n * n
            diag_parts.append(torch.diagonal(H).contiguous())
            d_off[k] = dn
            dn += n
        host_h16[n] = torch.cat(parts).cpu().pin_memory()
        dev_h16[n] = torch.empty_like(host_h16[n], device="cuda")
    host_d32 = torch.cat(diag_parts).cpu().pin_memory()
    dev_d32 = torch.empty_like(host_d32, device="cuda")
    dev_H = {k: torch.empty_like(wl.hess[k]) for k in keys}
    host_out = torch.empty(max(1, my_bytes if world == 1 else (sum(all_sizes) if rank == 0 else 0)),
                           dtype=torch.uint8).pin_memory()
    h2d = host_w.numel() * 2 + sum(v.numel() * 2 for v in host_h16.values()) + host_d32.numel() * 4
    d2h = sum(all_sizes) if rank == 0 else 0
    # every host-to-device copy goes out in order on one stream, so the link never waits for
    # a kernel; the Hessian decodes and the weight conversions run on high-priority streams
    # (they must not queue behind the fits and the factor chains) that wait for their copy
    xfer = torch.cuda.Stream()
    hcopy_stream = torch.cuda.Stream(priority=-1)
    conv_stream = torch.cuda.Stream(priority=-1)
    hs_ = nat.stream_ptr(torch, hcopy_stream)
    # the stored diagonal is exact float32 and the decoded H carries it unchanged, so the
    # host copy gives act order and damping without reading H back
    hd = host_d32.numpy().astype(np.float64)
    host_diag = {k: hd[d_off[k]:d_off[k] + int(wl.hess[k].shape[0])] for k in keys}
    # the weights travel in about twelve chunks cut at tensor boundaries; each chunk's round-1
    # fits start once that chunk is on the device and converted.  Chunks holding a tensor
    # without EF (token_embd: two fits, the largest fit work per byte) go first, so that the
    # chunk arriving last leaves little fit work behind it.
    names = [wl.uid(u) for u in wl.units]
    counts = [(u.r1 - u.r0) * wl.spec_by_name[u.name].n for u in wl.units]
    plain = {wl.uid(u) for u in wl.units if wl.spec_by_name[u.name].mode != "EF"}
    chunks, cur, acc, off = [], [], 0, 0
    target = max(1, sum(counts) // 12)
    for nm, c in zip(names, counts):
        if cur and (nm in plain) != any(x in plain for x in cur):
            chunks.append((off, off + acc, cur))
            off, cur, acc = off + acc, [], 0
        cur.append(nm)
        acc += c
        if acc >= target:
            chunks.append((off, off + acc, cur))
            off, cur, acc = off + acc, [], 0
    if cur:
        chunks.append((off, off + acc, cur))
    chunks.sort(key=lambda ch: (not any(x in plain for x in ch[2]), -(ch[1] - ch[0])))
    d2h_stream = torch.cuda.Stream()

    def step():
        # PCIe order: all diagonals (the fits' imatrix), the first weight chunk (token_embd:
        # its two fits keep the GPU busy from the first milliseconds), the Hessians largest
        # size first (the longest factor chain starts as soon as they are decoded), then the
        # remaining weight chunks; every chunk's fits wait only for that chunk.
        sizes = sorted(by_size, reverse=True)
        ready = {}

        def arrived():
            e = torch.cuda.Event()
            e.record(xfer)
            return e

        def hessians(ns):
            for n in ns:
                with torch.cuda.stream(xfer):
                    dev_h16[n].copy_(host_h16[n], non_blocking=True)
                hcopy_stream.wait_event(arrived())
                for k in by_size[n]:
                    nat.check(nat.lib().cp_hessian_decode(
                        dev_h16[n].data_ptr() + 2 * h_off[k], dev_d32.data_ptr() + 4 * d_off[k],
                        float(hscale[k]), n, nat.ptr(dev_H[k]), hs_), "hessian_decode")
                ready[n] = torch.cuda.Event()
                ready[n].record(hcopy_stream)

        staged = []

        def weights(part):
            for a, b, nms in part:
                with torch.cuda.stream(xfer):
                    dev_w16[a:b].copy_(host_w[a:b], non_blocking=True)
                conv_stream.wait_event(arrived())
                with torch.cuda.stream(conv_stream):
                    wl.x_flat[a:b].copy_(dev_w16[a:b])
                ev = torch.cuda.Event()
                ev.record(conv_stream)
                staged.append((ev, nms))

        cur_s = torch.cuda.current_stream()
        for st_ in (xfer, hcopy_stream, conv_stream):
            st_.wait_stream(cur_s)
        with torch.cuda.stream(xfer):
            dev_d32.copy_(host_d32, non_blocking=True)
        hcopy_stream.wait_event(arrived())
        with torch.cuda.stream(hcopy_stream):
            for k in wl.qw:
                wl.qw[k].copy_(dev_d32[d_off[k]:d_off[k] + wl.qw[k].numel()])
        qw_ready = torch.cuda.Event()   # the fits read these imatrix means
        qw_ready.record(hcopy_stream)
        cur_s.wait_event(qw_ready)
        weights(chunks[:1])
        hessians(sizes[:1])
        hessians(sizes[1:])
        weights(chunks[1:])
        hs = {k: dev_H[k] for k in wl.ef_keys}

        def copy_out(ev, _names):   # one GPU: the bytes leave while the statistics run
            d2h_stream.wait_event(ev)
            with torch.cuda.stream(d2h_stream):
                host_out[:my_bytes].copy_(flat[:my_bytes], non_blocking=True)

        enc.run(jobs, hs, {k: host_diag[k] for k in wl.ef_keys}, stats=True, outputs=outputs,
                inputs_event=staged, ready_events=ready, after_pack=copy_out if world == 1 else None)
        if world > 1:
            bufs = gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
            if rank == 0:
                off = 0
                for b in bufs:
                    host_out[off:off + b.numel()].copy_(b[:b.numel()], non_blocking=True)
                    off += b.numel()
        torch.cuda.synchronize()

    for _ in range(max(1, min(args.warmup, 2))):
        step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = (time.perf_counter() - t0) / args.steps
    if world > 1:
        t = torch.tensor([dt], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    return {"value": wl.total_params / dt / 1e6, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "seconds_per_step": dt,
            "path": "host float16 weights + stored-form Hessians -> device decode -> encode -> host bytes"}


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        import datetime
        import torch
        import torch.distributed as dist
        if args.impl == "reference":
            return reference_arm(args, rank, world)
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))
        try:
            return gpu_arm(args, rank, world, local_rank)
        finally:
            dist.destroy_process_group()
    if args.impl == "reference":
        return reference_arm(args, rank, world)
    return gpu_arm(args, rank, world, local_rank)


if __name__ == "__main__":
    sys.exit(main())
