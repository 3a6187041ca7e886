"""cp_xtx_accumulate (the tensor-core X^T X of Hessian collection, coldpress/hessians.py:
137-152) against a float64 product of the same activations, through the C ABI.

Tolerance.  The reference forms x.T @ x in float32 (`x.float()` first), so its own result
carries float32 matmul rounding.  Errors here are measured element-wise against the float64
product, scaled by sqrt(H_ii H_jj) (the Cauchy-Schwarz bound of sum |x_i x_j|), and the
tensor-core result must stay within 4x the error of torch's float32 matmul on the same
activations (floor 2^-22).  bf16 activations give exact float32 products; float32
activations are split into hi + lo bf16 (2^-17 relative remainder) and must also beat a
plain bf16 cast of the activations by 20x.  H must stay exactly symmetric and two runs must
give identical bits (the per-item partial tiles are summed in token order).  The shapes cover
the kernel's schedules: one pair tile cut over the SM pairs (d <= 256), whole rounds of pair
tiles plus a last round of sub-items (d = 3072, 4096), and several token splits per pair tile
(262144 x 1024).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

FLOOR = 2.0 ** -22


def _lib():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from perm_b200 import _native as nat
    return torch, nat, nat.lib()


def _acts(torch, T, d, seed, dtype):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    scales = torch.exp(torch.randn(d, device="cuda", generator=g))
    x = torch.randn(T, d, device="cuda", generator=g) * scales
    return x.to(dtype).contiguous()


def _run(torch, nat, L, x, H):
    T, d = x.shape
    dt = nat.CP_XTX_BF16 if x.dtype == torch.bfloat16 else nat.CP_XTX_F32
    nb = L.cp_xtx_workspace_bytes(dt, T, d)
    ws = torch.zeros(max(nb, 256), dtype=torch.uint8, device="cuda")
    s = nat.stream_ptr(torch)
    rc = L.cp_xtx_accumulate(dt, nat.ptr(x), T, d, nat.ptr(H), nat.ptr(ws), ws.numel(), s)
    assert rc == nat.CP_OK, nat.last_error()
    assert L.cp_xtx_status(nat.ptr(ws), s) == nat.CP_OK, nat.last_error()
    return H


def _err(H, ref, xtx):
    """max |H - ref| / sqrt(xtx_ii xtx_jj) over all elements."""
    dg = torch_sqrt_diag(xtx)
    return float(((H.double() - ref).abs() / (dg[:, None] * dg[None, :]).clamp_min(1e-300)).max())


def torch_sqrt_diag(xtx):
    return xtx.diagonal().clamp_min(0).sqrt()


@pytest.mark.parametrize("T,d", [(1, 128), (37, 8), (100, 136), (4096, 1024), (20000, 520), (3000, 3072),
                                 (777, 2048), (16384, 4096), (262144, 256), (262144, 1024)])
def test_xtx_bf16_matches_float64(T, d):
    torch, nat, L = _lib()
    x = _acts(torch, T, d, T * 31 + d, torch.bfloat16)
    H0 = torch.randn(d, d, device="cuda")
    H0 = (H0 + H0.T).contiguous()
    H = _run(torch, nat, L, x, H0.clone())
    xd = x.double()
    xtx = xd.T @ xd
    ref = H0.double() + xtx
    e32 = _err(H0 + x.float().T @ x.float(), ref, xtx)
    err = _err(H, ref, xtx)
    print(f"T={T} d={d}: tensor-core err {err:.3g}, torch float32 matmul err {e32:.3g}")
    assert err <= 4 * max(e32, FLOOR)
    assert torch.equal(H, H.T)
    H2 = _run(torch, nat, L, x, H0.clone())
    assert torch.equal(H, H2), "two runs differ"


@pytest.mark.parametrize("T,d", [(513, 256), (9000, 1024)])
def test_xtx_float32_keeps_float32_accuracy(T, d):
    torch, nat, L = _lib()
    x = _acts(torch, T, d, 7 + d, torch.float32)
    H = _run(torch, nat, L, x, torch.zeros(d, d, device="cuda"))
    xd = x.double()
    ref = xd.T @ xd
    err, e32 = _err(H, ref, ref), _err(x.T @ x, ref, ref)
    xb = x.to(torch.bfloat16).double()
    eb = _err(xb.T @ xb, ref, ref)
    print(f"T={T} d={d} float32: err {err:.3g}, torch float32 matmul err {e32:.3g}, bf16 cast err {eb:.3g}")
    assert err <= 4 * max(e32, FLOOR)
    assert eb > 20 * err
    assert torch.equal(H, H.T)


def test_xtx_accumulates_over_calls_and_python_wrapper():
    torch, nat, L = _lib()
    from perm_b200 import hessians
    d = 384
    xs = [_acts(torch, T, d, T, torch.bfloat16) for T in (64, 1000, 5)]
    H = torch.zeros(d, d, device="cuda")
    for x in xs:
        hessians.xtx_accumulate(x, H)
    hessians.xtx_status()
    ref = sum(x.double().T @ x.double() for x in xs)
    f32 = sum(x.float().T @ x.float() for x in xs)
    assert _err(H, ref, ref) <= 4 * max(_err(f32, ref, ref), FLOOR)
    # float16 input is widened to float32 (exactly representable as hi + lo)
    x16 = _acts(torch, 300, d, 3, torch.float16)
    H16 = hessians.xtx_accumulate(x16, torch.zeros(d, d, device="cuda"))
    ref16 = x16.double().T @ x16.double()
    assert _err(H16, ref16, ref16) <= 4 * max(_err(x16.float().T @ x16.float(), ref16, ref16), FLOOR)


def test_xtx_rejects_bad_shapes():
    torch, nat, L = _lib()
    from perm_b200 import hessians
    x = torch.zeros(4, 12, device="cuda", dtype=torch.bfloat16)
    with pytest.raises(ValueError):
        hessians.xtx_accumulate(x, torch.zeros(12, 12, device="cuda"))
    with pytest.raises(ValueError):
        hessians.xtx_accumulate(torch.zeros(4, 16, device="cuda", dtype=torch.bfloat16),
                                torch.zeros(8, 8, device="cuda"))
    ws = torch.zeros(256, dtype=torch.uint8, device="cuda")
    x = torch.zeros(64, 1024, device="cuda", dtype=torch.bfloat16)
    H = torch.zeros(1024, 1024, device="cuda")
    need = L.cp_xtx_workspace_bytes(nat.CP_XTX_BF16, 64, 1024)
    if need > 256:
        rc = L.cp_xtx_accumulate(nat.CP_XTX_BF16, nat.ptr(x), 64, 1024, nat.ptr(H), nat.ptr(ws), 256,
                                 nat.stream_ptr(torch))
        assert rc == nat.CP_ERR_WORKSPACE
    rc = L.cp_xtx_accumulate(nat.CP_XTX_BF16, nat.ptr(x), 0, 1024, nat.ptr(H), nat.ptr(ws), 256,
                             nat.stream_ptr(torch))
    assert rc == nat.CP_OK


def _tiny_llama(torch, dtype):
    from transformers import LlamaConfig, LlamaForCausalLM
    torch.manual_seed(0)
    cfg = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2,
                      num_attention_heads=4, num_key_value_heads=2, head_dim=64)
    return LlamaForCausalLM(cfg).to("cuda", dtype).eval()


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_collect_hessians_matches_reference_hook(dtype):
    """collect_hessians on a tiny Llama against the reference hook restated in float64."""
    torch, nat, L = _lib()
    from perm_b200 import hessians
    model = _tiny_llama(torch, getattr(torch, dtype))
    names = hessians.build_name_map(model, "llama", 2)
    ne0 = {g + ".weight": (model.get_submodule(m).in_features if hasattr(model.get_submodule(m), "in_features")
                           else model.get_submodule(m).embedding_dim) for m, g in names.items()}
    g = torch.Generator().manual_seed(1)
    batches = [torch.randint(0, 512, (2, 64), generator=g) for _ in range(3)]

    ref, rcnt = {}, {}
    hooks = []
    for m, gname in names.items():
        mod = model.get_submodule(m)
        if not isinstance(mod, torch.nn.Linear):
            continue

        def fn(mod, inp, out, gname=gname + ".weight"):
            x = inp[0].detach().reshape(-1, inp[0].shape[-1]).double()
            ref[gname] = ref.get(gname, 0) + x.T @ x
            rcnt[gname] = rcnt.get(gname, 0) + x.shape[0]
        hooks.append(mod.register_forward_hook(fn))
    with torch.inference_mode():
        for ids in batches:
            model(ids.cuda())
    for h in hooks:
        h.remove()

    got, unmapped = hessians.collect_hessians(model, batches, ne0, "llama", 2, log=lambda *a: None)
    assert set(got) == set(ref)
    for k, v in got.items():
        assert v["n"] == rcnt[k]
        r = ref[k].cpu().numpy()
        assert v["H"].dtype == np.float32 and v["H"].shape == r.shape
        dg = np.sqrt(np.clip(np.diag(r), 0, None))
        assert (np.abs(v["H"] - r) / np.maximum(dg[:, None] * dg[None, :], 1e-300)).max() <= 1e-5, k
    assert np.array_equal(got["blk.0.attn_q.weight"]["H"], got["blk.0.attn_k.weight"]["H"])
    solo, _ = hessians.collect_hessians(model, batches, ne0, "llama", 2, log=lambda *a: None, share_inputs=False)
    for k in got:
        assert np.array_equal(got[k]["H"], solo[k]["H"]), k


@pytest.mark.parametrize("dtype_name,T,d,skip", [("bf16", 4096, 512, 5), ("f32", 2048, 256, 70)])
def test_xtx_bounded_wait_runs_out_and_reports_timeout(dtype_name, T, d, skip):
    """The failure path of the bounded waits, made on the host: cp_xtx_inject_stall arms the
    next call so that its loader issues nothing for one 64-token step, and every wait gives up
    after 2 ms.  The kernel must stop, report CP_ERR_TIMEOUT through cp_xtx_status and leave
    the device usable: the next (unarmed) call on the same workspace is correct again."""
    torch, nat, L = _lib()
    dtype = torch.bfloat16 if dtype_name == "bf16" else torch.float32
    x = _acts(torch, T, d, 11, dtype)
    dt = nat.CP_XTX_BF16 if dtype_name == "bf16" else nat.CP_XTX_F32
    ws = torch.zeros(max(L.cp_xtx_workspace_bytes(dt, T, d), 256), dtype=torch.uint8, device="cuda")
    s = nat.stream_ptr(torch)
    assert L.cp_xtx_inject_stall(skip, 2_000_000) == nat.CP_OK
    H = torch.zeros(d, d, device="cuda")
    assert L.cp_xtx_accumulate(dt, nat.ptr(x), T, d, nat.ptr(H), nat.ptr(ws), ws.numel(), s) == nat.CP_OK
    rc = L.cp_xtx_status(nat.ptr(ws), s)
    assert rc == nat.CP_ERR_TIMEOUT, nat.last_error()
    assert "ran out" in nat.last_error()
    # the status word was cleared, nothing is left armed, and the device still computes
    H2 = _run(torch, nat, L, x, torch.zeros(d, d, device="cuda"))
    ref = x.double().T @ x.double()
    f32 = x.float().T @ x.float()
    assert _err(H2, ref, ref) <= 4 * max(_err(f32, ref, ref), FLOOR)
