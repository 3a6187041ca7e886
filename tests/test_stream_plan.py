"""Host logic of the memory-bounded batches (perm_b200.stream.plan) on the CPU: every job lands
in exactly one batch, in order; a Hessian's jobs stay together; batches respect the byte
budget unless a single group alone exceeds it."""
from dataclasses import dataclass

import pytest


@dataclass
class FakeJob:
    name: str
    mode: str
    hkey: str
    params: int


def _llama_like_jobs(layers=6):
    from perm_b200 import model
    specs = model.tensor_specs(model.MODELS["llama3-8b"], "q4_k_m_style")
    specs = [s for s in specs if not s.name.startswith("blk.") or int(s.name.split(".")[1]) < layers]
    return [FakeJob(s.name, s.mode, s.hkey, s.params) for s in specs], model.hessian_dims(specs)


@pytest.mark.parametrize("budget_gb", [5, 20, 40, 1000])
def test_plan_covers_jobs_in_order_and_keeps_groups(budget_gb):
    from perm_b200 import stream as stm
    jobs, dims = _llama_like_jobs()
    plan = stm.plan(jobs, dims, budget_gb * 1e9)
    flat = [j.name for b in plan for j in b]
    assert flat == [j.name for j in jobs]
    owner = {}
    for bi, b in enumerate(plan):
        for j in b:
            if j.mode == "EF":
                assert owner.setdefault(j.hkey, bi) == bi, f"{j.hkey} split across batches"
    for b in plan:
        keys = {j.hkey for j in b if j.mode == "EF"}
        cost = sum(j.params * stm.ef_bytes_per_param() for j in b if j.mode == "EF") + \
            sum(j.params * 0.1 for j in b if j.mode != "EF") + sum(stm.hessian_bytes(dims[k]) for k in keys)
        groups = len(keys) + sum(1 for j in b if j.mode != "EF")
        assert cost <= budget_gb * 1e9 or groups == 1
    if budget_gb == 1000:
        assert len(plan) == 1


def test_hessian_bytes_counts_h_workspace_and_u():
    from perm_b200 import _native as nat
    from perm_b200 import stream as stm
    n = 14336
    L = nat.lib()
    assert stm.hessian_bytes(n) == 8 * n * n + L.cp_factor_workspace_bytes(n) + L.cp_ef_u_bytes(n)
    assert stm.hessian_bytes(n) > 4e9
