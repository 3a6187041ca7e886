"""Host logic of collect_hessians (coldpress/hessians.py:85-183) on the CPU: name mapping,
token counts, input sharing between sibling projections and its per-batch verification.
The device product is replaced by torch's float32 matmul here, so the result must equal the
reference hook's arithmetic bit for bit."""
import numpy as np
import pytest
import torch


def _fake_accumulate(x, H, stream=None):
    H += x.float().T @ x.float()
    return H


@pytest.fixture
def host_hessians(monkeypatch):
    from perm_b200 import hessians
    monkeypatch.setattr(hessians, "xtx_accumulate", _fake_accumulate)
    return hessians


def _tiny_llama():
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=128, hidden_size=64, intermediate_size=128, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=16)
    return LlamaForCausalLM(cfg).eval()


def _ne0(model, names):
    out = {}
    for m, g in names.items():
        mod = model.get_submodule(m)
        out[g + ".weight"] = mod.in_features if isinstance(mod, torch.nn.Linear) else mod.embedding_dim
    return out


def _reference_hook_run(model, names, batches):
    """The reference hook's arithmetic: float32 x.T @ x summed per tensor, rows counted."""
    acc, cnt, hooks = {}, {}, []
    for m, g in names.items():
        mod = model.get_submodule(m)

        def fn(mod, inp, out, g=g + ".weight"):
            x = inp[0]
            if not torch.is_floating_point(x):
                return
            x = x.detach().reshape(-1, x.shape[-1]).float()
            if g not in acc:
                acc[g] = torch.zeros(x.shape[1], x.shape[1])
                cnt[g] = 0
            acc[g] += x.T @ x
            cnt[g] += x.shape[0]
        hooks.append(mod.register_forward_hook(fn))
    with torch.inference_mode():
        for ids in batches:
            model(ids if ids.dim() > 1 else ids.unsqueeze(0))
    for h in hooks:
        h.remove()
    return {g: {"H": acc[g].numpy(), "n": cnt[g]} for g in acc}


def test_collect_hessians_host_logic_matches_reference_hook(host_hessians):
    model = _tiny_llama()
    names = host_hessians.build_name_map(model, "llama", 2)
    ne0 = _ne0(model, names)
    g = torch.Generator().manual_seed(2)
    batches = [torch.randint(0, 128, (2, 16), generator=g) for _ in range(3)] + [torch.randint(0, 128, (16,), generator=g)]
    want = _reference_hook_run(model, names, batches)
    for share in (True, False):
        got, unmapped = host_hessians.collect_hessians(model, batches, ne0, "llama", 2, log=lambda *a: None,
                                                       share_inputs=share)
        assert set(got) == set(want)
        assert "token_embd.weight" not in got     # ids in, no Hessian
        for k in want:
            assert got[k]["n"] == want[k]["n"]
            assert np.array_equal(got[k]["H"], want[k]["H"]), (share, k)


def test_collect_hessians_layer_shard_and_mismatch(host_hessians):
    model = _tiny_llama()
    names = host_hessians.build_name_map(model, "llama", 2)
    ne0 = _ne0(model, names)
    batches = [torch.randint(0, 128, (1, 8))]
    got, _ = host_hessians.collect_hessians(model, batches, ne0, "llama", 2, layer_lo=1, layer_hi=2,
                                            log=lambda *a: None)
    assert got and all(k.startswith("blk.1.") for k in got)
    bad = dict(ne0)
    bad["blk.0.attn_q.weight"] = 32
    with pytest.raises(ValueError):
        host_hessians.collect_hessians(model, batches, bad, "llama", 2, log=lambda *a: None)


class _Attn(torch.nn.Module):
    """q and k read the same input on even calls and different inputs on odd calls."""

    def __init__(self):
        super().__init__()
        self.q_proj = torch.nn.Linear(16, 16, bias=False)
        self.k_proj = torch.nn.Linear(16, 16, bias=False)
        self.calls = 0

    def forward(self, x):
        y = self.q_proj(x)
        z = self.k_proj(x if self.calls % 2 == 0 else x * 2)
        self.calls += 1
        return y + z


class _Toy(torch.nn.Module):
    def __init__(self):
        super().__init__()
        self.attn = _Attn()

    def forward(self, ids):
        return self.attn(ids.float().reshape(-1, 16))


def test_collect_hessians_detects_sharing_that_breaks(host_hessians, monkeypatch):
    toy = _Toy()
    monkeypatch.setattr(host_hessians, "build_name_map",
                        lambda model, arch, n: {"attn.q_proj": "blk.0.attn_q", "attn.k_proj": "blk.0.attn_k"})
    ne0 = {"blk.0.attn_q.weight": 16, "blk.0.attn_k.weight": 16}
    batches = [torch.arange(32).reshape(2, 16) for _ in range(2)]
    with pytest.raises(RuntimeError, match="share_inputs=False"):
        host_hessians.collect_hessians(toy, batches, ne0, "llama", 1, log=lambda *a: None)
    toy.attn.calls = 0
    got, _ = host_hessians.collect_hessians(toy, batches, ne0, "llama", 1, log=lambda *a: None, share_inputs=False)
    x = torch.arange(32).reshape(2, 16).float()
    assert np.array_equal(got["blk.0.attn_q.weight"]["H"], (x.T @ x + x.T @ x).numpy())
    assert np.array_equal(got["blk.0.attn_k.weight"]["H"], (x.T @ x + (2 * x).T @ (2 * x)).numpy())
