"""Sharding of a whole-model encode across the GPUs of one node.

Work units are (tensor, row range): error-feedback rows are independent once U and the
per-row committed grid are known, and k-quant superblocks never straddle rows, so a tensor
can be split at any row boundary and its packed rows concatenated afterwards.  There is no
exchange during compute; the only collective is the gather of packed bytes (and the per-unit
error sums of the statistics) to rank 0.

Cost model (per unit, arbitrary but consistent units):
    EF:    sweep 2 * n_iter * rows * n^2/2 ordered updates + n_iter fits
    fit:   rows * n * passes(type, path), passes = candidate evaluations per element
    factor (2/3) n^3 FP64 flops, charged once per distinct Hessian per rank
Greedy LPT: units sorted by cost, each to the rank whose load (including any factorisation
it would newly need) grows least.  Units of one Hessian group are kept whole unless they
exceed a fair share, so U is usually computed once per node.
"""
import contextlib
from dataclasses import dataclass, field

# candidate evaluations per element of one fit (kquant.py: 1 + nstep+1 candidates for qkx,
# 19 for make_qx, ~6 for the Q3_K reference path), imatrix / reference path
FIT_PASSES = {("Q2_K", True): 38, ("Q2_K", False): 17, ("Q3_K", True): 19, ("Q3_K", False): 6,
              ("Q4_K", True): 38, ("Q4_K", False): 22, ("Q5_K", True): 38, ("Q5_K", False): 17,
              ("Q6_K", True): 19, ("Q6_K", False): 19}
# Relative weights, fitted to B200 times of every rank's share of the 4- and 8-way plans of
# the 0.6B model (one GPU per share, least squares over sweep updates, candidate evaluations
# and FP64 flops; residuals under 0.5 ms): one candidate-element evaluation of a fit costs
# about 20 ordered updates, one FP64 flop of the factorisation about one.
FIT_OP_WEIGHT = 20.0      # candidate-element evaluation relative to one ordered update
FACTOR_WEIGHT = 1.0       # FP64 flop relative to one ordered update
WRTN_FITS = 2.0           # fit passes charged to a weighted-RTN tensor (its fit and the stock baseline)


@dataclass
class UnitMeta:
    name: str
    ttype: str
    mode: str
    nrow: int
    n: int
    hkey: str = None
    imat: bool = True


@dataclass
class Unit:
    name: str
    r0: int
    r1: int
    cost: float


@dataclass
class Plan:
    world: int
    units: list = field(default_factory=list)        # per rank: list of Unit
    loads: list = field(default_factory=list)

    def rank_units(self, r):
        return self.units[r]


def unit_cost(m, rows, n_iter=2):
    fit = rows * m.n * FIT_PASSES.get((m.ttype, m.imat), 20) * FIT_OP_WEIGHT
    if m.mode == "EF":
        return n_iter * (rows * m.n * (m.n - 1) / 2.0) + n_iter * fit
    if m.mode == "wRTN(attn0-diag)":
        return WRTN_FITS * fit
    return fit


def factor_cost(n):
    return FACTOR_WEIGHT * (2.0 / 3.0) * float(n) ** 3


def make_plan(metas, world, n_iter=2, split_factor=2.0):
    """Split and assign units.  metas: list of UnitMeta.  Returns Plan."""
    plan = Plan(world, [[] for _ in range(world)], [0.0] * world)
    if world == 1:
        for m in metas:
            plan.units[0].append(Unit(m.name, 0, m.nrow, unit_cost(m, m.nrow, n_iter)))
        plan.loads[0] = sum(u.cost for u in plan.units[0])
        return plan
    total = sum(unit_cost(m, m.nrow, n_iter) for m in metas)
    fair = total / world
    cap = fair / split_factor
    groups = {}
    for m in metas:
        groups.setdefault(m.hkey if m.mode == "EF" else ("solo", m.name), []).append(m)
    items = []   # (cost, hkey or None, [(meta, r0, r1)])
    for key, ms in groups.items():
        gcost = sum(unit_cost(m, m.nrow, n_iter) for m in ms)
        hk = key if not isinstance(key, tuple) else None
        if gcost <= cap:
            items.append((gcost, hk, [(m, 0, m.nrow) for m in ms]))
            continue
        for m in ms:
            c = unit_cost(m, m.nrow, n_iter)
            pieces = max(1, int(-(-c // cap)))
            step = -(-m.nrow // pieces)
            for r0 in range(0, m.nrow, step):
                r1 = min(m.nrow, r0 + step)
                items.append((unit_cost(m, r1 - r0, n_iter), hk, [(m, r0, r1)]))
    items.sort(key=lambda t: -t[0])
    have = [set() for _ in range(world)]
    dims = {m.hkey: m.n for m in metas if m.hkey is not None}
    for cost, hk, parts in items:
        best, best_load = 0, None
        for r in range(world):
            extra = factor_cost(dims[hk]) if (hk is not None and hk not in have[r]) else 0.0
            load = plan.loads[r] + cost + extra
            if best_load is None or load < best_load:
                best, best_load = r, load
        plan.loads[best] = best_load
        if hk is not None:
            have[best].add(hk)
        for m, r0, r1 in parts:
            plan.units[best].append(Unit(m.name, r0, r1, unit_cost(m, r1 - r0, n_iter)))
    return plan


def gather_to_rank0(torch, dist, flat, sizes, rank, world):
    """Send each rank's flat uint8 buffer to rank 0 over NCCL; returns the list of received
    buffers on rank 0 (rank 0's own buffer first) and None elsewhere."""
    if world == 1:
        return [flat]
    if rank == 0:
        bufs = [flat] + [torch.empty(int(sizes[r]), dtype=torch.uint8, device=flat.device) for r in range(1, world)]
        ops = [dist.P2POp(dist.irecv, bufs[r], r) for r in range(1, world) if sizes[r] > 0]
        if ops:
            for req in dist.batch_isend_irecv(ops):
                req.wait()
        return bufs
    if sizes[rank] > 0:
        for req in dist.batch_isend_irecv([dist.P2POp(dist.isend, flat, 0)]):
            req.wait()
    return None


def unit_tensor(name):
    """Tensor name of a unit id `name[r0:r1]` (the name itself when it carries no row range)."""
    return name.split("[", 1)[0] if name.endswith("]") and "[" in name else name


def merge_unit_stats(stats):
    """Per-tensor statistics from per-unit ones ({unit id: stats dict with "err" and
    "err_stock", the weighted squared-error sums of the encode and of the stock baseline}):
    the sums of a tensor's row ranges add, so rel_err_vs_stock = sum(err) / sum(err_stock) - 1
    is the same number a single-device encode of the whole tensor reports (up to float64
    summation order)."""
    out = {}
    for name, st in stats.items():
        t = unit_tensor(name)
        o = out.setdefault(t, {"type": st.get("type"), "mode": st.get("mode"), "err": 0.0, "err_stock": 0.0})
        o["err"] += float(st["err"])
        o["err_stock"] += float(st["err_stock"])
    for o in out.values():
        o["rel_err_vs_stock"] = o["err"] / o["err_stock"] - 1 if o["err_stock"] else 0.0
    return out


def gather_stats_to_rank0(dist, stats, rank, world):
    """Per-unit statistics of every rank, merged per tensor on rank 0 (None elsewhere).  The
    error sums travel as Python objects through the process group (a few KB)."""
    if world == 1:
        return merge_unit_stats(stats)
    got = [None] * world if rank == 0 else None
    dist.gather_object(stats, got, dst=0)
    if rank != 0:
        return None
    allst = {}
    for d in got:
        allst.update(d)
    return merge_unit_stats(allst)


class HostGather:
    """One host buffer, in POSIX shared memory, that every rank of a node writes its packed
    bytes into, each over its own PCIe link.  Rank 0 then holds the whole model's bytes in host
    memory without a device-side gather and without one link carrying all of them (the
    alternative to gather_to_rank0 followed by rank 0's device-to-host copy).

    Rank 0 creates the segment (`sizes[r]` bytes per rank, in rank order) and the others attach
    to it by name.  With `register=True` every rank page-locks the mapping with the CUDA driver
    (cudaHostRegister), so copies into it can be asynchronous.  Raises OSError when /dev/shm
    has not the room (the caller then keeps the device gather); every rank makes the same
    decision, since rank 0 broadcasts it.  After each rank's copies have completed, `barrier()`
    tells rank 0 that `view` is whole.  `close()` releases the segment on every rank."""

    def __init__(self, torch, dist, sizes, rank, world, register=True):
        import os
        from multiprocessing import shared_memory
        self.torch, self.dist, self.rank, self.world = torch, dist, rank, world
        self.sizes = [int(v) for v in sizes]
        self.total = max(1, sum(self.sizes))
        self.off = sum(self.sizes[:rank])
        msg = [None]
        shm = None
        if rank == 0:
            try:
                st = os.statvfs("/dev/shm")
                if st.f_bavail * st.f_frsize < self.total + (64 << 20):
                    raise OSError("/dev/shm has not the room for the host gather")
                shm = shared_memory.SharedMemory(create=True, size=self.total)
                msg = [shm.name]
            except OSError as e:
                msg = ["!" + str(e)]
        dist.broadcast_object_list(msg, src=0)
        if msg[0].startswith("!"):
            raise OSError(msg[0][1:])
        if rank == 0:   # a step that raises before close() still leaves no segment behind
            import atexit
            atexit.register(HostGather._unlink_quietly, shm.name)
        ok = 1
        if rank != 0:
            try:
                shm = shared_memory.SharedMemory(name=msg[0])
            except OSError:
                shm, ok = None, 0
            else:
                try:   # the creating rank owns the segment: keep this process's tracker from unlinking it
                    from multiprocessing import resource_tracker
                    resource_tracker.unregister(shm._name, "shared_memory")
                except Exception:
                    pass
        self.shm = shm
        self.view = torch.frombuffer(shm.buf, dtype=torch.uint8)[:self.total] if shm is not None else None
        self.mine = self.view[self.off:self.off + self.sizes[rank]] if shm is not None else None
        self.registered = False
        if register and shm is not None:
            rc = int(torch.cuda.cudart().cudaHostRegister(self.view.data_ptr(), self.total, 0))
            self.registered = rc == 0
            ok = int(self.registered)
        # every rank takes the same path: an attach or a registration that failed anywhere
        # closes the buffer everywhere
        flag = torch.tensor([ok], dtype=torch.int32,
                            device="cuda" if dist.get_backend() == "nccl" else "cpu")
        dist.all_reduce(flag, op=dist.ReduceOp.MIN)
        if int(flag.item()) == 0:
            self.close()
            raise OSError("attaching or page-locking the host gather buffer failed on a rank")

    def barrier(self):
        self.dist.barrier()

    @staticmethod
    def _unlink_quietly(name):
        from multiprocessing import shared_memory
        try:
            seg = shared_memory.SharedMemory(name=name)
        except OSError:
            return   # already unlinked by close()
        seg.close()
        seg.unlink()

    def close_local(self):
        if self.registered:
            self.torch.cuda.cudart().cudaHostUnregister(self.view.data_ptr())
            self.registered = False
        self.view = self.mine = None
        if self.shm is not None:
            try:
                self.shm.close()
            except BufferError:   # a tensor over the buffer is still alive: unmapped at exit
                pass

    def close(self):
        """Every rank unmaps; rank 0 unlinks the segment once the others are done with it."""
        self.close_local()
        self.dist.barrier()
        if self.rank == 0 and self.shm is not None:
            self.shm.unlink()
        self.shm = None


class RankFailure(RuntimeError):
    """Another rank reported a failure between steps."""


class RankGuard:
    """Host-side failure detection between the steps of a multi-rank encode.

    A rank whose step raises writes its rank and error to the process group's store before
    leaving; every rank checks that key before it starts a step (and so before the step's
    collectives) and raises RankFailure naming the failed rank instead of entering a
    collective that would wait for it.  A rank that dies without reaching the store, or fails
    while the others are already inside a collective, is caught by the process group's
    timeout, which callers keep short.  No device work is involved: a failed rank leaves only
    between steps, with none of its kernels or collectives in flight."""

    def __init__(self, store, rank, world, key="perm_b200/failed"):
        self.store, self.rank, self.world, self.key = store, rank, world, key

    def failed(self):
        """(rank, message) of a reported failure, or None."""
        if not self.store.check([self.key]):
            return None
        v = self.store.get(self.key).decode(errors="replace")
        r, _, msg = v.partition(":")
        return int(r), msg

    def check(self):
        f = self.failed()
        if f is not None:
            raise RankFailure(f"rank {f[0]} failed: {f[1]}")

    def report(self, exc):
        try:
            self.store.set(self.key, f"{self.rank}:{type(exc).__name__}: {exc}"[:500])
        except Exception:   # the store itself may be gone; the timeout still bounds the others
            pass

    @contextlib.contextmanager
    def step(self):
        """with guard.step(): ... -- checks for an earlier failure first, reports this rank's."""
        self.check()
        try:
            yield
        except RankFailure:
            raise
        except BaseException as e:
            self.report(e)
            raise
