"""Sharding plan and the rank-0 gather (CPU; the gather runs as two gloo ranks)."""
import os

import numpy as np
import pytest


def _metas():
    from perm_b200 import model, shard
    specs = model.tensor_specs(model.MODELS["qwen3-0.6b"], "q2_k_mix")
    return specs, [shard.UnitMeta(s.name, s.ttype, s.mode, s.nrow, s.n, s.hkey, True) for s in specs]


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_plan_covers_every_row_once_and_balances(world):
    from perm_b200 import shard
    specs, metas = _metas()
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
