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
    # the second workload of the line: the Llama-3-8B-shaped Q4_K_M-style encode (BASELINE
    # config[4]), streamed through the device in batches of layers
    ap.add_argument("--no-gguf", action="store_true")
    ap.add_argument("--no-config2", action="store_true")
    ap.add_argument("--no-config4", action="store_true")
    ap.add_argument("--config4-model", default="llama3-8b")
    ap.add_argument("--config4-mixture", default="q4_k_m_style")
    ap.add_argument("--config4-tokens", type=int, default=131072)
    ap.add_argument("--config4-steps", type=int, default=2)
    ap.add_argument("--config4-warmup", type=int, default=3)
    ap.add_argument("--config4-budget-gb", type=float, default=0.0,
                    help="device bytes per batch (0: 30%% of the memory free once the inputs are resident)")
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


def bench_config(args, world):
    """The `config` of both arms' lines (the reference arm times a bounded sample of it)."""
    from perm_b200 import model
    specs = model.tensor_specs(model.MODELS[args.model], args.mixture)
    params = sum(s.params for s in specs)
    return {"workload": f"{args.model}-shaped whole-model EF encode, {args.mixture} "
                        f"({len(specs)} tensors, {params / 1e6:.1f} M params)",
            "mixture": args.mixture, "n_iter": 2, "damp": 0.01, "act_order": True,
            "hessian_tokens": args.hessian_tokens,
            "l2": "inputs (3 GB weights + float64 Hessians) are larger than L2; no flush",
            "parallelism": f"tensor/row-range shards over {world} GPU(s), NCCL gather of packed bytes"}


# ----------------------------------------------------------------------------- reference as-is

REF_DIR = os.path.join(ROOT, "baseline", "_ref")

# One worker of the as-is reference timing: imports coldpress from the unmodified install in
# baseline/_ref, builds its tensor's seeded inputs, waits for the common start time, then runs
# the reference's ef.ef_encode plus the statistics' stock roundtrip (ef.py:298) and prints its
# seconds.  argv: ref_dir, kind ("config0" | layer tensor index), seed, start_at (epoch s).
_REF_WORKER = r"""
import json, sys, time
import numpy as np
ref_dir, kind, seed, start_at = sys.argv[1], sys.argv[2], int(sys.argv[3]), float(sys.argv[4])
sys.path.insert(0, ref_dir)
from coldpress import ef, kquant as kq
rng = np.random.default_rng(seed)
if kind == "config0":
    nrow, n, tt = 3072, 1024, "Q2_K"
    W = (rng.standard_normal((nrow, n)) * 0.02).astype(np.float32)
    W[:, rng.choice(n, n // 100, replace=False)] *= 8.0
    T = 8192
else:
    shapes = [(2048, 1024, "Q2_K"), (1024, 1024, "Q2_K"), (1024, 1024, "Q3_K"), (1024, 2048, "Q3_K"),
              (3072, 1024, "Q2_K"), (3072, 1024, "Q2_K"), (1024, 3072, "Q3_K")]
    nrow, n, tt = shapes[int(kind)]
    W = (rng.standard_normal((nrow, n)) * 0.02).astype(np.float32)
    T = 8192
X = rng.standard_normal((T, n)).astype(np.float32) * rng.lognormal(0, 1, n).astype(np.float32)
H = (X.T.astype(np.float64) @ X.astype(np.float64)) / T
qw = np.diag(H).astype(np.float32)
while time.time() < start_at:
    time.sleep(0.01)
t0 = time.time()
ef.ef_encode(W, tt, qw, H, n_iter=2, damp=0.01, act_order=True)
kq.roundtrip(W, tt, qw)
t1 = time.time()
print(json.dumps({"params": int(W.size), "seconds": t1 - t0, "late": t0 - start_at}))
"""


def reference_available():
    return os.path.isdir(os.path.join(REF_DIR, "coldpress"))


def _ref_workers(kinds, seed, threads_each, setup_s):
    """Run one as-is reference worker per entry of `kinds` at once; returns their records."""
    env = dict(os.environ)
    if threads_each is not None:
        for v in ("OPENBLAS_NUM_THREADS", "OMP_NUM_THREADS", "MKL_NUM_THREADS"):
            env[v] = str(threads_each)
    start_at = time.time() + setup_s
    procs = [subprocess.Popen([sys.executable, "-c", _REF_WORKER, REF_DIR, str(k), str(seed + i), repr(start_at)],
                              stdout=subprocess.PIPE, stderr=subprocess.PIPE, env=env, text=True)
             for i, k in enumerate(kinds)]
    out = []
    for p in procs:
        o, e = p.communicate(timeout=900)
        if p.returncode != 0:
            raise RuntimeError(f"reference worker failed: {e.strip()[-300:]}")
        out.append(json.loads(o.strip().splitlines()[-1]))
    return out


def run_reference_as_is(seed):
    """BASELINE's two CPU numbers for the reference itself, unmodified (baseline/_ref):
    (i) one process with default BLAS threads on one config[0] tensor (3072 x 1024 Q2_K EF);
    (ii) one single-threaded process per tensor of layer 0 of the 0.6B model (7 tensors,
    25.2 M params), all at once on the host cores (OPENBLAS_NUM_THREADS=1)."""
    if not reference_available():
        return {"unavailable": "the reference is not installed in baseline/_ref"}
    nt = cpu_threads()
    one = _ref_workers(["config0"], seed, None, 3.0)[0]
    par = _ref_workers([str(i) for i in range(7)], seed, 1, 10.0)
    wall = max(r["seconds"] + r["late"] for r in par)
    params = sum(r["params"] for r in par)
    return {"reference_as_is": {"value": one["params"] / one["seconds"] / 1e6, "unit": UNIT, "cores": nt,
                                "kind": "reference", "seconds": one["seconds"],
                                "sample": "coldpress.ef.ef_encode + stock roundtrip, unmodified, one process "
                                          "(default BLAS threads), one config[0] tensor 3072x1024 Q2_K"},
            "reference_parallel": {"value": params / wall / 1e6, "unit": UNIT, "cores": min(nt, 7),
                                   "kind": "reference", "seconds": wall,
                                   "sample": "coldpress.ef.ef_encode + stock roundtrip, unmodified, one "
                                             "single-threaded process per tensor of layer 0 (7 tensors, "
                                             "25.2 M params), run at once"}}


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


def run_cpu_baseline_on_workload(torch, wl, outputs, rows_big=64):
    """The CPU port timed on a bounded sample of the GPU workload itself, which doubles as the
    bench's parity check: layer 0's seven tensors (the timed sample) plus the first rows of
    output.weight and token_embd.weight, with the same weights and Hessians as the device run,
    encoded by the CPU oracle (a restatement of ef.py / kquant.py) and compared byte for byte
    with the packed bytes the last timed step left on the device (rows are independent, so a
    row slice of a tensor encodes to the same bytes as those rows of the whole tensor)."""
    from oracle import oracle as orc
    orc.build()
    nt = cpu_threads()
    items = []
    for u in wl.units:
        sp = wl.spec_by_name[u.name]
        if sp.name.startswith("blk.0."):
            items.append((u, sp, slice(0, u.r1 - u.r0), True))
        elif sp.name in ("output.weight", "token_embd.weight"):
            items.append((u, sp, slice(0, min(rows_big, u.r1 - u.r0)), False))
    host_h = {}
    n_params, dt = 0, 0.0
    checked, same_bytes, min_codes = 0, 0, 1.0
    for u, sp, rs, timed in items:
        uid = wl.uid(u)
        W = wl.x[uid][rs].cpu().numpy()
        if sp.hkey not in host_h:
            host_h[sp.hkey] = wl.hess[sp.hkey].cpu().numpy()
        H = host_h[sp.hkey]
        qw = wl.diags[sp.hkey].astype(np.float32)
        t0 = time.perf_counter()
        if sp.mode == "EF":
            want, _ = orc.ef_encode(W, sp.ttype, qw, H, n_iter=2, act_order=True, nthreads=nt)
            orc.roundtrip(W, sp.ttype, qw)   # the statistics' stock baseline (ef.py:298)
        else:   # token_embd: weighted RTN with the attn0 diagonal (ef.py:280-285), plus its baseline
            want = orc.quantize(sp.ttype, W, qw, nt)
            orc.roundtrip(W, sp.ttype, None)
        if timed:
            dt += time.perf_counter() - t0
            n_params += W.size
        got = outputs[uid][rs].cpu().numpy()
        checked += 1
        same_bytes += int(np.array_equal(got, want))
        codes = float(np.mean(orc.codes(sp.ttype, got, *W.shape) == orc.codes(sp.ttype, want, *W.shape)))
        min_codes = min(min_codes, codes)
    return {"value": n_params / dt / 1e6, "unit": UNIT, "cores": nt, "kind": "port", "seconds": dt,
            "sample": "layer 0 of the bench workload itself (7 tensors, 25.2 M params, the same weights and "
                      "262144-token Hessians): EF n_iter 2 (numpy LAPACK factor + C oracle fits and sweeps, "
                      "all host threads) plus the stock-baseline roundtrip",
            "parity": {"tensors_checked": checked, "bytes_identical_tensors": same_bytes,
                       "min_codes_identical": min_codes,
                       "sample": f"layer 0's 7 tensors whole + the first {rows_big} rows of output.weight and "
                                 "token_embd.weight, CPU oracle vs the last timed step's device bytes"}}


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
            "config": bench_config(args, world),
            "cpu_baseline": {"value": value, "unit": UNIT, "cores": nt, "kind": "port",
                             "sample": "bounded sample of the workload per step: layer 0 of the Qwen3-0.6B-shaped "
                                       "model (7 tensors, 25.2 M params), EF n_iter 2 + stock roundtrip through "
                                       "the CPU restatement of the reference (numpy LAPACK factor, C fits and "
                                       "sweeps, all host threads)"},
            "e2e": {"value": value, "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


# ----------------------------------------------------------------------------- GPU arm

class Workload:
    """Inputs of this rank's units, resident on the device.  stored=True keeps the Hessians in
    the reference's storage form (float16 H / hscale + float32 diagonal, perm_b200.stream) for
    a model encoded in batches (decoded per batch inside the step) instead of as float64."""

    def __init__(self, torch, args, rank, world, model_name=None, mixture=None, tokens=None, stored=False):
        from perm_b200 import model, shard
        self.torch = torch
        model_name = model_name or args.model
        mixture = mixture or args.mixture
        tokens = tokens or args.hessian_tokens
        self.model_name, self.mixture, self.tokens, self.stored_mode = model_name, mixture, tokens, stored
        cfg = model.MODELS[model_name]
        self.specs = model.tensor_specs(cfg, mixture)
        self.spec_by_name = {s.name: s for s in self.specs}
        metas = [shard.UnitMeta(s.name, s.ttype, s.mode, s.nrow, s.n, s.hkey, s.mode != "wRTN(attn0-diag)")
                 for s in self.specs]
        self.plan = shard.make_plan(metas, world)
        self.units = self.plan.units[rank]
        self.total_params = sum(s.params for s in self.specs)
        dims = model.hessian_dims(self.specs)
        self.dims = dims
        need = set()
        for u in self.units:
            sp = self.spec_by_name[u.name]
            need.add(sp.hkey)
        self.hess, self.diags, self.stored = {}, {}, {}
        for k in sorted(need):
            H = model.synth_hessian(torch, dims[k], k, args.seed, "cuda", tokens=tokens)
            if stored:
                from perm_b200 import stream as stm
                self.stored[k] = stm.store_hessian(torch, H)
                self.diags[k] = self.stored[k].diag_host
                del H
            else:
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
        factor_flops = sum((2.0 / 3.0) * float(self.dims[k]) ** 3 for k in self.ef_keys)
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


def make_guard(dist, rank, world):
    """RankGuard over the process group's store (N > 1): a rank whose step raises reports it,
    the others stop before their next step's collectives.  A no-op context at N = 1."""
    import contextlib
    if world == 1:
        class _Solo:
            def step(self):
                return contextlib.nullcontext()
        return _Solo()
    from perm_b200.shard import RankGuard
    return RankGuard(dist.distributed_c10d._get_default_store(), rank, world)


def roofline_record(prof, alg, steps, clk):
    """Roofline of the dominant kernel, the error-feedback sweep, from this rank's algorithmic
    work and the live CUDA-event time of its launches (the sweep leads the serialised device
    time of a step).  The sweep is bound by ordered FP32 arithmetic, so the headline fraction
    is 2 unfused FP32 operations per ordered update against the FP32 lane rate (148 SMs x 128
    lanes x the SM clock sampled during the timed region; nominal: MEASURED_PEAKS.json has no
    FP32 figure).  Its HBM view (algorithmic bytes and the DRAM traffic per launch against the
    measured copy bandwidth) and the k-quant fit's and the FP64 factor's own rooflines are
    kept beside it."""
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    hbm = float(peaks.get("hbm_gbs", 6650.0))
    hbm_src = "measured (MEASURED_PEAKS.json hbm_gbs)" if "hbm_gbs" in peaks else "fallback 6650 GB/s"
    per_step = {c: (prof[c][0] / steps, prof[c][1] / steps) for c in prof}
    sm_mhz = clk.get("sm_mhz") or 1965.0
    fp32_peak = 148 * 128 * sm_mhz * 1e6 / 1e12   # T lane-ops/s: FADD/FMUL/FFMA one lane-op each
    fp32_src = f"nominal: 148 SMs x 128 FP32 lanes x {sm_mhz:.0f} MHz (sampled SM clock)"
    sw_ms, sw_l = per_step["sweep"]
    sw_l = max(1.0, sw_l)
    out = {"kernel": "ef_sweep", "bound": "fp32_alu", "unit": "T fp32 lane-ops/s", "peak": fp32_peak,
           "peak_source": fp32_src, "work": "2 unfused FP32 ops per ordered update",
           "ms_per_step": sw_ms, "launches_per_step": sw_l,
           "classes_ms_per_step": {c: round(per_step[c][0], 4) for c in per_step}}
    if sw_ms > 0:
        out["achieved"] = 2.0 * alg["sweep_updates"] / (sw_ms / 1e3) / 1e12
        out["frac"] = out["achieved"] / fp32_peak
        # DRAM bytes of one sweep launch: ncu (dram__bytes_read.sum + dram__bytes_write.sum) of
        # the second step's first sweep launch of the default 0.6B workload on one B200
        # measured 36.77 GB (31.37 read + 5.40 written) for 425.1 G ordered updates, 0.08649
        # bytes per update; per launch here = that rate x this rank's updates per round (the
        # error re-reads, the larger part, grow like the updates: n^2/32 bytes per row and
        # round against n^2/2 updates)
        traffic = 0.08649 * alg["sweep_updates"] / sw_l
        alg_bytes = alg["sweep_bytes"] / sw_l
        gbs = alg["sweep_bytes"] / (sw_ms / 1e3) / 1e9
        out["traffic"] = traffic
        out["traffic_unit"] = "DRAM bytes per launch (ncu rate, scaled by this rank's updates)"
        out["hbm"] = {"achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": gbs / hbm, "peak_source": hbm_src,
                      "algorithmic_bytes_per_launch": alg_bytes, "traffic": traffic,
                      "traffic_over_algorithmic": traffic / alg_bytes if alg_bytes else None}
    fit_ms = per_step["fit"][0]
    if fit_ms > 0:
        ach = 20.0 * alg["fit_evals"] / (fit_ms / 1e3) / 1e12
        out["fit"] = {"kernel": "kquant fit+pack", "bound": "fp32_alu", "achieved": ach, "peak": fp32_peak,
                      "unit": "T fp32 lane-ops/s", "frac": ach / fp32_peak,
                      "work": "~20 ops per candidate-element evaluation",
                      "hbm_gbs": alg["fit_bytes"] / (fit_ms / 1e3) / 1e9, "ms_per_step": fit_ms}
    fac_ms = per_step["factor"][0]
    if fac_ms > 0 and alg["factor_flops"] > 0:
        ach = alg["factor_flops"] / (fac_ms / 1e3) / 1e12
        out["factor"] = {"kernel": "fp64 factor (mma.sync f64)", "bound": "fp64_tensor", "achieved": ach,
                         "peak": 37.0, "unit": "FP64 TFLOP/s", "frac": ach / 37.0,
                         "peak_source": "measured back-to-back mma.sync f64 loop on this part (probe)",
                         "work": "(2/3) n^3 per factorisation; event spans overlap the fits, so a lower bound",
                         "ms_per_step": fac_ms}
    return out


def gpu_arm(args, rank, world, local_rank):
    import torch
    import torch.distributed as dist
    from perm_b200 import _native as nat
    from perm_b200.encoder import Encoder
    from perm_b200.shard import gather_stats_to_rank0, gather_to_rank0

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

    guard = make_guard(dist, rank, world)

    def step():
        with guard.step():
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

    roofline = roofline_record(prof, wl.algorithmic(), args.steps, clk)
    total_params, n_tensors = wl.total_params, len(wl.specs)
    merged = gather_stats_to_rank0(dist, st, rank, world)   # every rank's units, per tensor

    # the CPU port on a sample of this workload, checked against the bytes the last timed step
    # left on the device (before the e2e runs below overwrite the weights with float16 values)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = run_cpu_baseline_on_workload(torch, wl, outputs)

    e2e = None
    if not args.no_e2e:
        e2e = measure_e2e(torch, dist, args, wl, enc, jobs, outputs, flat, my_bytes, all_sizes, rank, world)

    gguf_rec = None
    if world == 1 and not args.no_gguf:
        gguf_rec = measure_gguf(torch, args, wl)

    cpu_ref = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            cpu_ref = run_reference_as_is(args.seed)
        except (RuntimeError, subprocess.TimeoutExpired, ValueError) as e:
            cpu_ref = {"reference_as_is": {"unavailable": str(e)[:200]}}
        cpu.update(cpu_ref)

    big = None
    if not args.no_config4:
        total_params = wl.total_params
        del wl, jobs, outputs, flat, enc
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        big = measure_streamed(torch, dist, args, rank, world, local_rank)
        wl = None

    xtx = None
    if not args.no_config2:
        xtx = measure_xtx(torch, dist, args, rank, world, local_rank)

    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": UNIT, "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "whole_model_seconds": ms / 1e3,
                "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
                "data": "synthetic (random-init N(0,0.02) weights, synthetic X^T X Hessians)",
                "config": bench_config(args, world),
                "gpu_launches": int(launches), "roofline": roofline, "clocks": clk, "e2e": e2e,
                "cpu_baseline": cpu, "stats_median_rel_err_vs_stock": float(np.median(
                    [v["rel_err_vs_stock"] for v in merged.values()])) if merged else None,
                "stats_tensors": len(merged) if merged else 0,
                "whole_model_seconds_gguf": gguf_rec,
                "config4": big, "config2": xtx}
        print(json.dumps(line), flush=True)
    return 0


def measure_gguf(torch, args, wl):
    """Whole-model seconds through the file formats (N = 1): the same 0.6B-shaped model written
    to local disk as the reference's encode inputs -- a float16 GGUF of the weights, a target
    GGUF of the Q2_K mixture, one compressed Hessian npz per tensor in the reference's storage
    form (hessians.py:185-207) and an imatrix GGUF holding diag(H) -- then encoded by
    perm_b200.ef.encode_gguf (the drop-in for ef.py:223-317), which reads, decodes, encodes
    and re-emits the GGUF.  One warm-up run, then one timed run; the files sit in the page
    cache (written just before).  Returns the record of the bench line."""
    import concurrent.futures as cf
    import shutil
    import tempfile
    import gguf
    from gguf import GGUFWriter
    from perm_b200 import ef, gguf_io, kquant as kq
    t0 = time.perf_counter()
    tmp = tempfile.mkdtemp(prefix="perm_b200_gguf_")
    try:
        f16p, tgtp, imp, outp = (os.path.join(tmp, n) for n in ("f16.gguf", "target.gguf", "imatrix.gguf",
                                                                 "out.gguf"))
        hdir = os.path.join(tmp, "hessians")
        os.makedirs(hdir)
        specs = [wl.spec_by_name[u.name] for u in wl.units]
        xs = {wl.uid(u): wl.x[wl.uid(u)] for u in wl.units}
        wf = GGUFWriter(f16p, "qwen3")
        wt = GGUFWriter(tgtp, "qwen3")
        for w_ in (wf, wt):
            w_.add_uint32("qwen3.block_count", 28)
            w_.add_string("general.name", "synthetic qwen3-0.6b-shaped")
        for u, sp in zip(wl.units, specs):
            x16 = xs[wl.uid(u)].to(torch.float16).cpu().numpy()
            wf.add_tensor(sp.name, x16)
            nb = kq.row_bytes(sp.ttype, sp.n)
            wt.add_tensor(sp.name, np.zeros((sp.nrow, nb), np.uint8), raw_shape=(sp.nrow, nb),
                          raw_dtype=getattr(gguf.GGMLQuantizationType, sp.ttype))
        for w_ in (wf, wt):
            w_.write_header_to_file()
            w_.write_kv_data_to_file()
            w_.write_tensors_to_file()
            w_.close()
        wi = GGUFWriter(imp, "imatrix")
        for sp in specs:
            if sp.mode == "EF":
                wi.add_tensor(sp.name + ".in_sum2", (wl.diags[sp.hkey] * 1000.0).astype(np.float32))
                wi.add_tensor(sp.name + ".counts", np.array([1000.0], np.float32))
        wi.write_header_to_file()
        wi.write_kv_data_to_file()
        wi.write_tensors_to_file()
        wi.close()
        # one npz per tensor with a Hessian (q/k/v and gate/up hold the same matrix), written
        # as the reference's collector writes them, on all host threads
        host_h = {k: (wl.hess[k] * wl.tokens).float().cpu().numpy() for k in wl.hess}
        todo = [(sp.name, host_h[sp.hkey]) for sp in specs if sp.mode == "EF"]
        with cf.ThreadPoolExecutor(max_workers=cpu_threads()) as ex:
            list(ex.map(lambda t: gguf_io.save_hessians({t[0]: {"H": t[1], "n": wl.tokens}}, hdir), todo))
        del host_h
        setup_s = time.perf_counter() - t0
        sizes = {"f16_gguf_bytes": os.path.getsize(f16p), "target_gguf_bytes": os.path.getsize(tgtp),
                 "hessian_npz_bytes": sum(os.path.getsize(os.path.join(hdir, f)) for f in os.listdir(hdir)),
                 "hessian_files": len(os.listdir(hdir))}
        quiet = lambda *_: None  # noqa: E731
        ef.encode_gguf(f16p, tgtp, hdir, outp, imatrix_path=imp, log=quiet)
        runs = []
        for _ in range(2):   # best of two timed runs (host file work varies run to run)
            tm = {}
            torch.cuda.synchronize()
            st = ef.encode_gguf(f16p, tgtp, hdir, outp, imatrix_path=imp, log=quiet, timings=tm)
            runs.append(tm)
        tm = min(runs, key=lambda r: r["wall_s"])
        rec = {"seconds": tm["wall_s"], "value": wl.total_params / tm["wall_s"] / 1e6, "unit": UNIT,
               "read_s": tm["read_s"], "device_s": tm["device_s"], "write_s": tm["write_s"],
               "h2d_bytes": tm["h2d_bytes"], "d2h_bytes": tm["d2h_bytes"], "batches": tm["batches"],
               "tensors": tm["tensors"], "out_gguf_bytes": os.path.getsize(outp), "setup_seconds": setup_s,
               "timed_runs_seconds": [round(r["wall_s"], 3) for r in runs],
               "page_cache": "warm (files written just before the runs)",
               "path": "perm_b200.ef.encode_gguf: GGUF/npz read (reader thread) -> float16 weights and "
                       "stored-form Hessians to the device -> decode, factor, EF encode -> GGUF re-emit",
               "stats_median_rel_err_vs_stock": float(np.median([v["rel_err_vs_stock"] for v in st.values()]))}
        rec.update(sizes)
        return rec
    finally:
        shutil.rmtree(tmp, ignore_errors=True)


def measure_streamed(torch, dist, args, rank, world, local_rank):
    """the Llama-3-8B-shaped model (32 layers, hidden 4096, 32 q / 8 kv
    heads x 128, ffn 14336, vocab 128256; 8.03 B parameters, 129 Hessians up to d = 14336 from
    131072 synthetic tokens) EF-encoded into the Q4_K_M-style mixture.  The weights (float32)
    and the Hessians in storage form (float16 / hscale + float32 diagonal) are resident; one
    step decodes every Hessian, factorises it, and encodes every tensor, in memory-bounded
    batches of whole Hessian groups (Encoder.run_stream), then (N > 1) gathers the packed
    bytes to rank 0.  Returns the `config4` record of the bench line (rank 0), or None."""
    from perm_b200 import _native as nat
    from perm_b200 import stream as stm
    from perm_b200.encoder import Encoder
    from perm_b200.shard import gather_stats_to_rank0, gather_to_rank0
    t_setup = time.perf_counter()
    torch.cuda.reset_peak_memory_stats()
    wl = Workload(torch, args, rank, world, model_name=args.config4_model, mixture=args.config4_mixture,
                  tokens=args.config4_tokens, stored=True)
    jobs = wl.jobs()
    sizes = wl.out_bytes()
    my_bytes = int(sum(sizes))
    flat = torch.empty(max(1, my_bytes), dtype=torch.uint8, device="cuda")
    outputs, off = {}, 0
    for u, sz, j in zip(wl.units, sizes, jobs):
        rows = u.r1 - u.r0
        outputs[j.name] = flat[off:off + sz].view(rows, sz // rows)
        off += sz
    if world > 1:
        t = torch.tensor([my_bytes], dtype=torch.int64, device="cuda")
        g = [torch.zeros(1, dtype=torch.int64, device="cuda") for _ in range(world)]
        dist.all_gather(g, t)
        all_sizes = [int(v.item()) for v in g]
    else:
        all_sizes = [my_bytes]
    torch.cuda.synchronize()
    free, _total = torch.cuda.mem_get_info()
    budget = args.config4_budget_gb * 1e9 if args.config4_budget_gb > 0 else 0.30 * free
    job_batches = stm.plan(jobs, wl.dims, budget)
    enc = Encoder(n_iter=2, damp=0.01, act_order=True)
    dec = torch.cuda.Stream(priority=-1)
    setup_s = time.perf_counter() - t_setup

    guard = make_guard(dist, rank, world)

    def step():
        with guard.step():
            _, st = enc.run_stream(stm.batches(torch, job_batches, wl.stored, outputs, dec), stats=True)
            if world > 1:
                gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
        return st

    if world > 1:
        dist.barrier()
    for _ in range(max(1, args.config4_warmup)):
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
    for _ in range(args.config4_steps):
        st = step()
    t_end.record()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    nat.profile_enable(False)
    launches = (nat.lib().cp_launch_count() - launches0) // max(1, args.config4_steps)
    prof = nat.profile_collect()
    clk = clocks.stop()
    ms = t_start.elapsed_time(t_end) / args.config4_steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = wl.total_params / (ms / 1e3) / 1e6
    roof = roofline_record(prof, wl.algorithmic(), args.config4_steps, clk)
    peak_gb = torch.cuda.max_memory_allocated() / 1e9
    merged = gather_stats_to_rank0(dist, st, rank, world)
    e2e = None
    if not args.no_e2e:
        e2e = streamed_e2e(torch, dist, args, wl, job_batches, outputs, flat, my_bytes, all_sizes, rank, world,
                           guard, enc)
    rec = None
    if rank == 0:
        rec = {"workload": f"{args.config4_model}-shaped whole-model EF encode, {args.config4_mixture} "
                           f"({len(wl.specs)} tensors, {wl.total_params / 1e6:.1f} M params)",
               "metric": METRIC.replace("(Q2_K)", "(Q4_K_M-style)"), "value": value, "unit": UNIT,
               "ms_per_step": ms, "whole_model_seconds": ms / 1e3, "steps": args.config4_steps,
               "warmup": max(1, args.config4_warmup), "n_gpus": world, "hessian_tokens": args.config4_tokens,
               "batches_per_step": len(job_batches), "batch_budget_gb": round(budget / 1e9, 2),
               "resident": "float32 weights + storage-form Hessians (float16/hscale + float32 diagonal); "
                           "each batch's Hessians decoded to float64 inside the step",
               "l2": "inputs (32 GB weights at N=1) are larger than L2; no flush",
               "gpu_launches": int(launches), "roofline": roof, "clocks": clk,
               "peak_device_gb_rank0": round(peak_gb, 1), "setup_seconds": round(setup_s, 1),
               "stats_median_rel_err_vs_stock": float(np.median([v["rel_err_vs_stock"] for v in merged.values()]))
               if merged else None, "stats_tensors": len(merged) if merged else 0, "e2e": e2e}
    del enc, outputs, flat, jobs, wl
    torch.cuda.synchronize()
    torch.cuda.empty_cache()
    return rec


def streamed_e2e(torch, dist, args, wl, job_batches, outputs, flat, my_bytes, all_sizes, rank, world, guard, enc):
    """config[4] end to end through host buffers: every step uploads each batch's float16
    weights and its Hessians in storage form (float16 bits / hscale + float32 diagonal, which
    is also the imatrix) from pinned host memory on a copy stream, widens and decodes them on
    the device, encodes the batch (Encoder.run_stream: the next batch's uploads and factor
    chains overlap the current batch's sweeps) and copies each finished batch's packed bytes
    back to pinned host memory; at N > 1 rank 0 gathers the other ranks' bytes over NCCL and
    copies them out too.  Wall time per step (host clock around synchronised steps), max over
    ranks."""
    from perm_b200 import _native as nat
    from perm_b200.encoder import Job, StreamBatch
    from perm_b200.shard import HostGather, gather_to_rank0
    host_w = {}
    for b in job_batches:
        for j in b:
            h = torch.empty(tuple(j.x.shape), dtype=torch.float16, pin_memory=True)
            h.copy_(j.x.to(torch.float16))
            host_w[j.name] = h
    def spec_hkey(j):   # the Hessian whose diagonal a job uses (token_embd: blk.0's q/k/v input)
        return wl.spec_by_name[j.name.split("[", 1)[0]].hkey

    keys = sorted({spec_hkey(j) for b in job_batches for j in b if spec_hkey(j) is not None})
    host_h, d_off, dn = {}, {}, 0
    for k in keys:
        sh = wl.stored[k]
        h = torch.empty(tuple(sh.h16.shape), dtype=torch.float16, pin_memory=True)
        h.copy_(sh.h16)
        host_h[k] = (h, float(sh.hscale), sh.d)
        d_off[k] = dn
        dn += sh.d
    host_d32 = torch.empty(max(1, dn), dtype=torch.float32, pin_memory=True)
    for k in keys:
        host_d32[d_off[k]:d_off[k] + wl.stored[k].d].copy_(wl.stored[k].diag32)
    dev_d32 = torch.empty_like(host_d32, device="cuda")
    # N > 1: each batch's bytes go over the rank's own link into one shared host buffer that rank
    # 0 reads (HostGather); without room in /dev/shm, the NCCL gather and rank 0's copy instead
    hg, hg_note = None, None
    if world > 1:
        try:
            hg = HostGather(torch, dist, all_sizes, rank, world)
        except OSError as e:
            hg_note = str(e)
    host_out = torch.empty(max(1, my_bytes if world == 1 else (sum(all_sizes) if rank == 0 and hg is None else 0)),
                           dtype=torch.uint8, pin_memory=True)
    h2d = sum(h.numel() * 2 for h in host_w.values()) + sum(v[0].numel() * 2 for v in host_h.values()) + dn * 4
    d2h = sum(all_sizes) if rank == 0 else 0
    copy_s, work_s, d2h_s = torch.cuda.Stream(), torch.cuda.Stream(priority=-1), torch.cuda.Stream()
    main = torch.cuda.current_stream()
    base = flat.data_ptr()

    def gen():
        with torch.cuda.stream(copy_s):   # every diagonal first: the imatrix of every fit
            dev_d32.copy_(host_d32, non_blocking=True)
        got_d32 = torch.cuda.Event()
        got_d32.record(copy_s)
        work_s.wait_event(got_d32)
        main.wait_event(got_d32)
        for jobs in job_batches:
            hs, diags, ready = {}, {}, {}
            for k in sorted({j.hkey for j in jobs if j.mode == "EF"}, key=lambda k: -host_h[k][2]):
                h, hscale, d = host_h[k]
                with torch.cuda.stream(copy_s):
                    h16 = torch.empty((d, d), dtype=torch.float16, device="cuda")
                    h16.copy_(h, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_s)
                work_s.wait_event(ev)
                with torch.cuda.stream(work_s):
                    H = torch.empty((d, d), dtype=torch.float64, device="cuda")
                nat.check(nat.lib().cp_hessian_decode(nat.ptr(h16), dev_d32.data_ptr() + 4 * d_off[k], hscale, d,
                                                      nat.ptr(H), nat.stream_ptr(torch, work_s)), "hessian_decode")
                h16.record_stream(work_s)
                done = torch.cuda.Event()
                done.record(work_s)
                ready[d] = done
                hs[k] = H
                diags[k] = wl.stored[k].diag_host
            staged, new_jobs = [], []
            for j in jobs:
                with torch.cuda.stream(copy_s):
                    x16 = torch.empty(tuple(j.x.shape), dtype=torch.float16, device="cuda")
                    x16.copy_(host_w[j.name], non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(copy_s)
                work_s.wait_event(ev)
                with torch.cuda.stream(work_s):
                    x = x16.float()
                x16.record_stream(work_s)
                x.record_stream(main)
                done = torch.cuda.Event()
                done.record(work_s)
                staged.append((done, [j.name]))
                hk = spec_hkey(j)
                qw = dev_d32[d_off[hk]:d_off[hk] + host_h[hk][2]] if hk is not None else None
                if j.mode == "EF":
                    new_jobs.append(Job(j.name, j.ttype, j.mode, x, qw, hk))
                else:   # token_embd: the attn0 diagonal as fit weights, unit statistics weights
                    new_jobs.append(Job(j.name, j.ttype, j.mode, x, None, None, fit_w=qw))
            yield StreamBatch(new_jobs, hs, diags, {j.name: outputs[j.name] for j in jobs}, staged, ready)

    def on_batch(b, raws, st):
        dst = hg.mine if hg is not None else host_out
        with torch.cuda.stream(d2h_s):
            for j in b.jobs:
                o = outputs[j.name]
                a = o.data_ptr() - base
                dst[a:a + o.numel()].copy_(o.view(-1), non_blocking=True)

    def step():
        with guard.step():
            enc.run_stream(gen(), stats=True, on_batch=on_batch if (world == 1 or hg is not None) else None)
            if world > 1 and hg is None:
                bufs = gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
                if rank == 0:
                    off = 0
                    with torch.cuda.stream(d2h_s):
                        d2h_s.wait_stream(main)
                        for bb in bufs:
                            host_out[off:off + bb.numel()].copy_(bb[:bb.numel()], non_blocking=True)
                            off += bb.numel()
            torch.cuda.synchronize()
            if hg is not None:
                hg.barrier()   # every rank's bytes are in rank 0's host buffer

    step()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.config4_steps):
        step()
    dt = (time.perf_counter() - t0) / args.config4_steps
    if world > 1:
        t = torch.tensor([dt], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        dt = float(t.item())
    out = {"value": wl.total_params / dt / 1e6, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h), "seconds_per_step": dt, "steps": args.config4_steps, "warmup": 1,
           "path": "host float16 weights + storage-form Hessians -> per-batch uploads, device decode -> "
                   "streamed encode -> host bytes"}
    if world > 1:
        out["d2h_path"] = ("each rank's bytes, batch by batch, over its own link into one shared host buffer read "
                           "by rank 0" if hg is not None else f"NCCL gather to rank 0, then rank 0's copy ({hg_note})")
    if hg is not None:   # outside the timed region: the host buffer against a device gather
        bufs = gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
        if rank == 0:
            ref = torch.cat([bb[:bb.numel()].cpu() for bb in bufs])
            out["host_gather_identical_to_device_gather"] = bool(torch.equal(ref, hg.view[:ref.numel()]))
            del ref
        del bufs
        hg.close()
    return out


def measure_xtx(torch, dist, args, rank, world, local_rank):
    """Hessian accumulation (the hook arithmetic of hessians.py:137-152,
    H = x^T x in float32) for the hooked Linear inputs of 28 Qwen3-0.6B-shaped layers, four
    distinct inputs per layer (q/k/v share d = 1024, attn_output d = 2048, gate/up share
    d = 1024, ffn_down d = 3072), 262144 bf16 tokens each (N(0, 1) x per-channel log-normal
    scales), through cp_xtx_accumulate on the tensor cores.  The 112 (layer, input) units are
    spread over the ranks by cost (d^2, greedy), and at N > 1 rank 0 gathers every rank's
    float32 [d, d] results over NCCL inside the step.  One bf16 activation matrix per distinct
    d stays resident (0.5 - 1.6 GB each, larger than L2), so each unit re-reads it from HBM."""
    from perm_b200 import _native as nat
    from perm_b200 import hessians
    from perm_b200.shard import gather_to_rank0
    T = args.hessian_tokens
    units = [(layer, kind, d) for layer in range(28)
             for kind, d in (("qkv", 1024), ("o", 2048), ("gateup", 1024), ("down", 3072))]
    loads, mine = [0.0] * world, [[] for _ in range(world)]
    for u in sorted(units, key=lambda u: -u[2]):
        r = min(range(world), key=lambda i: loads[i])
        loads[r] += float(u[2]) ** 2
        mine[r].append(u)
    my = mine[rank]
    sizes = [sum(d * d * 4 for _, _, d in mine[r]) for r in range(world)]
    flat = torch.empty(max(1, sizes[rank] // 4), dtype=torch.float32, device="cuda")
    Hs, off = [], 0
    for _, _, d in my:
        Hs.append(flat[off:off + d * d].view(d, d))
        off += d * d
    X = {}
    g = torch.Generator(device="cuda")
    g.manual_seed(args.seed * 31 + 7)
    for d in sorted({u[2] for u in units}):
        scales = torch.exp(torch.randn(d, generator=g, device="cuda"))
        X[d] = torch.empty((T, d), dtype=torch.bfloat16, device="cuda")
        for t0 in range(0, T, 32768):
            X[d][t0:t0 + 32768] = (torch.randn((min(32768, T - t0), d), generator=g, device="cuda") *
                                   scales).to(torch.bfloat16)
    flops = sum(2.0 * T * d * d for _, _, d in units)
    guard = make_guard(dist, rank, world)

    def step():
        with guard.step():
            flat.zero_()
            for (_, _, d), H in zip(my, Hs):
                hessians.xtx_accumulate(X[d], H)
            if world > 1:
                gather_to_rank0(torch, dist, flat.view(torch.uint8)[:sizes[rank]], sizes, rank, world)

    if world > 1:
        dist.barrier()
    for _ in range(args.warmup):
        step()
    hessians.xtx_status()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    clocks = ClockSampler(local_rank)
    clocks.start()
    nat.profile_enable(True)
    t_start, t_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t_start.record()
    for _ in range(args.steps):
        step()
    t_end.record()
    torch.cuda.synchronize()
    nat.profile_enable(False)
    clk = clocks.stop()
    prof = nat.profile_collect()
    hessians.xtx_status()
    if world > 1:
        dist.barrier()
    ms = t_start.elapsed_time(t_end) / args.steps
    if world > 1:
        t = torch.tensor([ms], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    kms = prof["other"][0] / args.steps   # the X^T X launches (this rank)
    my_flops = sum(2.0 * T * d * d for _, _, d in my)

    def executed(d):   # tensor-core flops of one unit: 256 x 256 pair tiles on or below the diagonal
        nT = -(-d // 256)
        return 2.0 * T * 256 * 256 * (nT * (nT + 1) // 2)
    my_exec = sum(executed(d) for _, _, d in my)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    # the timed region is a long run of back-to-back tensor-core work, so the power-capped
    # sustained figure is the denominator; the burst fraction rides along
    burst = float(peaks.get("bf16_tflops", 1590.0))
    peak = float(peaks.get("bf16_tflops_sustained", 1400.0))
    del X, flat, Hs
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    ach = my_exec / (kms / 1e3) / 1e12 if kms > 0 else None
    ach_alg = my_flops / (kms / 1e3) / 1e12 if kms > 0 else None
    return {"workload": "28 Qwen3-0.6B-shaped layers x 4 distinct Linear inputs (d 1024, 2048, 1024, 3072), "
                        f"{T} bf16 tokens each: H = x^T x in float32",
            "ms_per_step": ms, "seconds_per_step": ms / 1e3, "tflops_whole_job": flops / (ms / 1e3) / 1e12,
            "tokens_per_s_per_input": 112 * T / (ms / 1e3), "steps": args.steps, "warmup": args.warmup,
            "n_gpus": world, "units_rank0": len(my),
            "parallelism": "(layer, input) units by cost over the ranks, NCCL gather of the float32 [d, d] "
                           "results to rank 0 inside the step" if world > 1 else "one GPU",
            "roofline": {"kernel": "xtx_pair_kernel (tcgen05.mma.cta_group::2 kind::f16, TMEM accumulators)",
                         "bound": "tensor",
                         "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak if ach else None,
                         "peak_burst": burst, "frac_of_burst": ach / burst if ach else None,
                         "work": "tensor-core flops executed: 2 T x 256 x 256 per pair tile on or below the diagonal "
                                 "(H is symmetric, so about 55 % of a dense 2 T d^2)",
                         "algorithmic_equivalent_tflops": ach_alg,
                         "peak_source": "measured (MEASURED_PEAKS.json bf16_tflops_sustained: back to back under "
                                        "the power cap, like this timed region)" if "bf16_tflops_sustained" in peaks
                         else "fallback 1400 TFLOP/s sustained", "ms_per_step": kms},
            "clocks": clk}


def measure_e2e(torch, dist, args, wl, enc, jobs, outputs, flat, my_bytes, all_sizes, rank, world):
    """Same encode through host buffers: weights as float16 (the GGUF source dtype) and Hessians
    in the reference's storage form (float16 / hscale + exact float32 diagonal) copied from
    pinned memory every step, packed bytes copied back to pinned memory."""
    from perm_b200 import _native as nat
    from perm_b200.shard import HostGather, gather_to_rank0
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
    # N > 1: every rank copies its packed bytes over its own link into one shared host buffer
    # (HostGather) that rank 0 reads; without room in /dev/shm, the NCCL gather to rank 0 and
    # rank 0's copy of all the bytes instead
    hg, hg_note = None, None
    if world > 1:
        try:
            hg = HostGather(torch, dist, all_sizes, rank, world)
        except OSError as e:
            hg_note = str(e)
    host_out = torch.empty(max(1, my_bytes if world == 1 else (sum(all_sizes) if rank == 0 and hg is None else 0)),
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

        def copy_out(ev, _names):   # the bytes leave while the statistics run
            d2h_stream.wait_event(ev)
            with torch.cuda.stream(d2h_stream):
                dst = hg.mine if hg is not None else host_out[:my_bytes]
                dst.copy_(flat[:my_bytes], non_blocking=True)

        enc.run(jobs, hs, {k: host_diag[k] for k in wl.ef_keys}, stats=True, outputs=outputs,
                inputs_event=staged, ready_events=ready,
                after_pack=copy_out if (world == 1 or hg is not None) else None)
        if world > 1 and hg is None:
            bufs = gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
            if rank == 0:
                off = 0
                for b in bufs:
                    host_out[off:off + b.numel()].copy_(b[:b.numel()], non_blocking=True)
                    off += b.numel()
        torch.cuda.synchronize()
        if hg is not None:
            hg.barrier()   # every rank's bytes are in rank 0's host buffer

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
    out = {"value": wl.total_params / dt / 1e6, "unit": UNIT, "h2d_bytes_per_step": int(h2d),
           "d2h_bytes_per_step": int(d2h), "seconds_per_step": dt,
           "path": "host float16 weights + stored-form Hessians -> device decode -> encode -> host bytes"}
    if world > 1:
        out["d2h_path"] = ("each rank's bytes over its own link into one shared host buffer read by rank 0"
                           if hg is not None else f"NCCL gather to rank 0, then rank 0's copy ({hg_note})")
    if hg is not None:   # outside the timed region: the host buffer against a device gather
        bufs = gather_to_rank0(torch, dist, flat[:my_bytes], all_sizes, rank, world)
        if rank == 0:
            ref = torch.cat([b[:b.numel()].cpu() for b in bufs])
            out["host_gather_identical_to_device_gather"] = bool(torch.equal(ref, hg.view[:ref.numel()]))
        hg.close()
    return out


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
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
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
