"""Sharding plan and the rank-0 gather (CPU; the gather runs as two gloo ranks)."""
import os

import numpy as np
import pytest


def _metas(model_name="qwen3-0.6b", mixture="q2_k_mix"):
    from perm_b200 import model, shard
    specs = model.tensor_specs(model.MODELS[model_name], mixture)
    return specs, [shard.UnitMeta(s.name, s.ttype, s.mode, s.nrow, s.n, s.hkey, True) for s in specs]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("model_name,mixture", [("qwen3-0.6b", "q2_k_mix"), ("llama3-8b", "q4_k_m_style")])
def test_plan_covers_every_row_once_and_balances(world, model_name, mixture):
    from perm_b200 import shard
    specs, metas = _metas(model_name, mixture)
    plan = shard.make_plan(metas, world)
    rows = {s.name: np.zeros(s.nrow, np.int32) for s in specs}
    for r in range(world):
        for u in plan.units[r]:
            rows[u.name][u.r0:u.r1] += 1
    assert all((v == 1).all() for v in rows.values())
    loads = np.array(plan.loads)
    if world > 1:
        assert loads.max() / loads.mean() < 1.10, loads / loads.mean()


def test_plan_keeps_hessian_groups_together_when_small():
    from perm_b200 import shard
    specs, metas = _metas()
    plan = shard.make_plan(metas, 4)
    owner = {}
    for r in range(4):
        for u in plan.units[r]:
            owner.setdefault(u.name, set()).add(r)
    # q/k/v of a layer share a Hessian and are small: one rank computes their factor
    for layer in range(28):
        qkv = set().union(*(owner[f"blk.{layer}.attn_{x}.weight"] for x in "qkv"))
        assert len(qkv) == 1


def _gather_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from perm_b200.shard import gather_to_rank0
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        sizes = [5, 0, 7][:world]
        flat = torch.arange(sizes[rank], dtype=torch.uint8) + 10 * rank
        dist.barrier()
        bufs = gather_to_rank0(torch, dist, flat, sizes, rank, world)
        if rank == 0:
            out.put([b.tolist() for b in bufs])
    finally:
        dist.destroy_process_group()


def test_gather_to_rank0_with_gloo_ranks():
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_gather_worker, args=(r, 3, port, q)) for r in range(3)]
    for p in procs:
        p.start()
    got = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got == [[0, 1, 2, 3, 4], [], [20, 21, 22, 23, 24, 25, 26]]


def test_merge_unit_stats_adds_row_range_sums():
    from perm_b200.shard import merge_unit_stats, unit_tensor
    assert unit_tensor("output.weight[0:100]") == "output.weight"
    assert unit_tensor("blk.0.attn_q.weight") == "blk.0.attn_q.weight"
    st = {"output.weight[0:10]": {"type": "Q6_K", "mode": "EF", "err": 1.0, "err_stock": 2.0},
          "output.weight[10:30]": {"type": "Q6_K", "mode": "EF", "err": 3.0, "err_stock": 2.0},
          "blk.0.ffn_up.weight[0:3072]": {"type": "Q2_K", "mode": "EF", "err": 9.0, "err_stock": 10.0}}
    m = merge_unit_stats(st)
    assert set(m) == {"output.weight", "blk.0.ffn_up.weight"}
    assert m["output.weight"]["rel_err_vs_stock"] == 4.0 / 4.0 - 1
    assert abs(m["blk.0.ffn_up.weight"]["rel_err_vs_stock"] + 0.1) < 1e-12


def _init(rank, world, port, timeout_s):
    import datetime
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=timeout_s))
    return dist


def _stats_worker(rank, world, port, out):
    dist = _init(rank, world, port, 60)
    try:
        from perm_b200.shard import gather_stats_to_rank0
        mine = {f"output.weight[{10 * rank}:{10 * rank + 10}]": {"type": "Q6_K", "mode": "EF",
                                                                 "err": float(rank + 1), "err_stock": 2.0}}
        m = gather_stats_to_rank0(dist, mine, rank, world)
        if rank == 0:
            out.put(m)
    finally:
        dist.destroy_process_group()


def _spawn(target, world, extra=()):
    import socket
    import torch.multiprocessing as mp
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=target, args=(r, world, port, q) + tuple(extra)) for r in range(world)]
    for p in procs:
        p.start()
    return procs, q


def test_stats_gather_merges_every_rank():
    procs, q = _spawn(_stats_worker, 3)
    m = q.get(timeout=120)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert abs(m["output.weight"]["rel_err_vs_stock"] - (6.0 / 6.0 - 1)) < 1e-12


def _host_gather_worker(rank, world, port, out):
    dist = _init(rank, world, port, 60)
    try:
        import torch
        from perm_b200.shard import HostGather
        sizes = [5, 0, 7]
        hg = HostGather(torch, dist, sizes, rank, world, register=False)
        for step in range(2):   # two steps into the same buffer, as in a timed loop
            hg.mine.copy_(torch.full((sizes[rank],), 10 * step + rank + 1, dtype=torch.uint8))
            hg.barrier()
            if rank == 0:
                out.put(hg.view.tolist())
            hg.barrier()   # rank 0 has read this step before anyone writes the next
        hg.close()
    finally:
        dist.destroy_process_group()


def test_host_gather_assembles_every_rank_in_shared_memory():
    """HostGather: each rank writes its bytes into one shared host buffer (ragged sizes, an
    empty rank included); after the barrier rank 0 sees them in rank order, step after step."""
    procs, q = _spawn(_host_gather_worker, 3)
    got = [q.get(timeout=120) for _ in range(2)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for step in range(2):
        assert got[step] == [10 * step + 1] * 5 + [10 * step + 3] * 7


def _failing_worker(rank, world, port, out, fail_rank, fail_step):
    """Steps of one all-reduce each under a RankGuard; `fail_rank` raises between steps."""
    import time
    import torch
    dist = _init(rank, world, port, 5)
    from perm_b200.shard import RankFailure, RankGuard
    guard = RankGuard(dist.distributed_c10d._get_default_store(), rank, world)
    t0 = time.time()
    outcome = "completed"
    try:
        for step in range(6):
            with guard.step():
                if rank == fail_rank and step == fail_step:
                    raise ValueError("injected host failure")
                t = torch.ones(4)
                dist.all_reduce(t)
                time.sleep(0.05)
    except RankFailure as e:
        outcome = f"RankFailure: {e}"
    except ValueError as e:
        outcome = f"raised: {e}"
    except Exception as e:  # the process group's timeout ended a collective
        outcome = f"collective error: {type(e).__name__}"
    out.put((rank, outcome, time.time() - t0))
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def test_a_failing_rank_ends_the_others_without_a_hang():
    """One gloo rank raises between steps: it reports through the store, and every other rank
    ends with an error (RankFailure before its next step, or the short process-group timeout
    of a collective it had already entered) well within the bound, instead of hanging."""
    world, fail_rank = 3, 1
    procs, q = _spawn(_failing_worker, world, (fail_rank, 2))
    res = {}
    for _ in range(world):
        r, outcome, dt = q.get(timeout=120)
        res[r] = (outcome, dt)
    for p in procs:
        p.join(timeout=60)
        if p.exitcode is None:
            p.kill()
    assert res[fail_rank][0].startswith("raised: injected")
    for r in range(world):
        if r == fail_rank:
            continue
        outcome, dt = res[r]
        assert outcome.startswith("RankFailure: rank 1 failed") or outcome.startswith("collective error"), outcome
        assert dt < 30.0
