"""The whole-model forward around the blocks (model.py:1028-1116: input
embedding, text projection, timestep embedding chain, blocks, output norm and
projection) run by NativeWanModel against the fp32 CPU oracle
(oracle/wan_model.py, pinned to the reference source by
tests/golden/model_cases.pt), in action and latent mode, plus the device
flow-match step against the oracle scheduler.

Gate: the block gate of tests/blockutil.py: cosine >= 0.9999 and |err| <=
2e-2 plus half a bf16 ulp per bf16 rounding of the compared value (one for
the model's bf16 output; one per update for the bf16 sample of the
flow-match loop).
"""
import copy
import sys
from pathlib import Path

import pytest
import torch

from blockutil import assert_parity
from oracle import wan_model as om
from wam_ops import _lib
from wam_ops.model import NativeActionDenoiser, NativeWanModel
from wam_ops.scheduler import FlowMatchScheduler

sys.path.insert(0, str(Path(__file__).resolve().parent / "golden"))
from make_model_golden import CFG  # noqa: E402

pytestmark = pytest.mark.gpu


def _oracle_model(seed=11):
    torch.manual_seed(seed)
    m = om.WanTransformer3DModel(**CFG).eval()
    with torch.no_grad():
        for name, p in m.named_parameters():
            if name.endswith("scale_shift_table"):
                p.copy_(torch.randn_like(p) / p.shape[-1] ** 0.5)
            elif "norm" in name and name.endswith("weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p))
            elif "norm" in name and name.endswith("bias"):
                p.copy_(0.1 * torch.randn_like(p))
            elif name.endswith("weight"):
                p.copy_(torch.randn_like(p) * 0.05)
            else:
                p.copy_(0.05 * torch.randn_like(p))
            p.copy_(p.bfloat16().float())
    return m


def _to_device(m):
    """Reference dtype policy: fp32 for the modulation tables, norms and the
    timestep embedder (_keep_in_fp32_modules, model.py:812-825), bf16 else."""
    g = copy.deepcopy(m)
    keep32 = ("scale_shift_table", "norm1", "norm2", "norm3", "time_embedder")
    for name, p in g.named_parameters():
        fp32 = any(k in name for k in keep32)
        p.data = p.data.to(device="cuda", dtype=torch.float32 if fp32 else torch.bfloat16).contiguous()
    return g


def _inputs(action_mode, seed):
    g = torch.Generator().manual_seed(seed)
    from oracle import wan_block as ob
    if action_mode:
        B, f, h, w = 2, 8, 4, 1
        x = torch.randn(B, CFG["action_dim"], f, h, w, generator=g)
        grid = ob.get_mesh_id(f, h, w, 0, action=True)
    else:
        B, f, h, w = 1, 2, 8, 8
        x = torch.randn(B, CFG["in_channels"], f, h, w, generator=g)
        grid = ob.get_mesh_id(f, h // 2, w // 2, 0)
    x = x.bfloat16().float()
    text = torch.randn(B, 16, CFG["text_dim"], generator=g).bfloat16().float()
    steps = torch.rand(B, f, generator=g) * 1000
    return {"noisy_latents": x, "text_emb": text, "grid_id": grid[None], "timesteps": steps}


def _cuda(d, dtype=torch.bfloat16):
    return {k: (v.cuda().to(dtype) if k in ("noisy_latents", "text_emb") else v.cuda()) for k, v in d.items()}


@pytest.mark.parametrize("action_mode", [True, False])
@pytest.mark.parametrize("prepared", [False, True])
def test_model_forward(cuda_device, action_mode, prepared):
    m = _oracle_model()
    inp = _inputs(action_mode, 50 + int(action_mode))
    with torch.no_grad():
        ref = m(inp, action_mode=action_mode)
        rb = _to_device(m)(_cuda(inp), action_mode=action_mode)
    dev = _to_device(m)
    nm = NativeWanModel(dev)
    with torch.no_grad():
        if prepared:
            nm.prepare_context(_cuda(inp)["text_emb"])
        out = nm(_cuda(inp), action_mode=action_mode)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert out.shape == ref.shape and out.dtype == torch.bfloat16
    s = assert_parity(out, ref, rb, name=f"model {'action' if action_mode else 'latent'}"
                                          f"{' prepared' if prepared else ''}")
    print("model", "action" if action_mode else "latent", "prepared" if prepared else "", s)


@pytest.mark.parametrize("kw,n", [({"shift": 5.0, "sigma_min": 0.0, "extra_one_step": True}, 10), ({}, 50)])
def test_flow_step(cuda_device, kw, n):
    so, sn = om.FlowMatchScheduler(**kw), FlowMatchScheduler(**kw)
    so.set_timesteps(n)
    sn.set_timesteps(n)
    assert torch.equal(so.sigmas, sn.sigmas) and torch.equal(so.timesteps, sn.timesteps)
    g = torch.Generator().manual_seed(n)
    sample, v = torch.randn(4, 1000, generator=g), torch.randn(4, 1000, generator=g)
    for t in sn.timesteps[::3]:
        want = so.step(v, t, sample)
        got = sn.step(v.cuda(), t, sample.cuda())
        torch.cuda.synchronize()
        assert torch.allclose(got.cpu(), want, rtol=1e-6, atol=1e-6)
    x = sample.cuda().bfloat16()
    sn.step_(v.cuda().bfloat16(), sn.timesteps[0], x)
    ref = (sample.bfloat16().float() + v.bfloat16().float() * (float(so.sigmas[1]) - float(so.sigmas[0])))
    assert torch.allclose(x.float().cpu(), ref, rtol=2 ** -8, atol=1e-2)


def test_action_chunk_denoiser(cuda_device):
    """Three flow-match updates of an action chunk with a KV history: the
    captured graph equals the eager native loop bit for bit, and follows the
    fp32 oracle loop (model + scheduler) within the block gate."""
    m = _oracle_model(seed=12)
    inp = _inputs(True, 77)
    pool, hist = 96, 64
    g = torch.Generator().manual_seed(3)
    for blk in m.blocks:
        blk.attn1.init_kv_cache("pos", pool, 2, 128, "cpu", torch.float32, 2)
        c = blk.attn1.attn_caches["pos"]
        c["k"].copy_(torch.randn(c["k"].shape, generator=g).bfloat16().float())
        c["v"].copy_(torch.randn(c["v"].shape, generator=g).bfloat16().float())
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist) // 32
    kw = {"shift": 5.0, "sigma_min": 0.0, "extra_one_step": True}
    so, sn = om.FlowMatchScheduler(**kw), FlowMatchScheduler(**kw)
    so.set_timesteps(3)
    sn.set_timesteps(3)

    def run_ref(model, sched, x, dev):
        for t in sched.timesteps:
            d = dict(inp, noisy_latents=x, timesteps=torch.full_like(inp["timesteps"], float(t)))
            d = _cuda(d) if dev else d
            v = model(d, action_mode=True)
            B, C = x.shape[:2]
            v = v.reshape(B, -1, C).permute(0, 2, 1).reshape(x.shape)
            x = sched.step(v.float(), t, x.float()).to(x.dtype)
        return x

    def dev_copy():
        d = _to_device(m)
        for blk in d.blocks:
            c = blk.attn1.attn_caches["pos"]
            for k in list(c):
                c[k] = c[k].to(device="cuda", dtype=torch.bfloat16 if k in ("k", "v") else c[k].dtype)
        return d

    with torch.no_grad():
        ref = run_ref(m, so, inp["noisy_latents"], False)
        rb = run_ref(dev_copy(), so, inp["noisy_latents"].cuda().bfloat16(), True)
    dev = dev_copy()
    nm = NativeWanModel(dev)
    with torch.no_grad():
        nm.prepare_context(_cuda(inp)["text_emb"])
        x0 = _cuda(inp)["noisy_latents"]
        eager = x0.clone()
        for t in sn.timesteps:
            v = nm({"noisy_latents": eager, "grid_id": inp["grid_id"].cuda(),
                    "timesteps": torch.full((2, 8), float(t), device="cuda")}, action_mode=True)
            B, C = eager.shape[:2]
            _lib.check(_lib.load().wamb_flow_step_cl(eager.data_ptr(), 0, v.data_ptr(), 0, B, C, 32,
                                                     sn.delta(t), _lib.stream_ptr()))
        den = NativeActionDenoiser(nm, sn)
        den.capture(x0, inp["grid_id"].cuda())
        out = den.run(x0).clone()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.equal(out, eager)
    # The bf16 sample is re-rounded after each of the three updates (the fp32
    # oracle loop keeps it fp32), so the allowance is three half-ulps.
    s = assert_parity(out, ref, rb, roundings=3, name="action chunk, 3 updates")
    print("action chunk", s)


def test_kv_lifecycle_prefill_denoise_commit(cuda_device):
    """The KV-cache lifecycle at model level (model.py:547-593, 667-686): two
    video chunks prefilled in latent mode with update_cache=2 (written into
    the pool under chunk ids), an action denoise with update_cache=0 over that
    history (the mask restored after it), a prediction committed with
    update_cache=1, clear_pred_cache (Attention.clear_pred_cache), and a
    final read-only action denoise. Every native output follows the fp32
    oracle model within the block gate and the cache metadata (id, mask,
    is_pred) matches the oracle's bit for bit after every call."""
    from oracle import wan_block as ob
    m = _oracle_model(seed=31)
    pool = 160
    for blk in m.blocks:
        blk.attn1.init_kv_cache("pos", pool, 2, 128, "cpu", torch.float32, 1)
        c = blk.attn1.attn_caches["pos"]
        c["k"].zero_()
        c["v"].zero_()

    def dev_copy():
        d = _to_device(m)
        for blk in d.blocks:
            c = blk.attn1.attn_caches["pos"]
            for k in list(c):
                c[k] = c[k].to(device="cuda", dtype=torch.bfloat16 if k in ("k", "v") else c[k].dtype)
        return d

    rb_model, dev = dev_copy(), dev_copy()
    nm = NativeWanModel(dev)
    g = torch.Generator().manual_seed(8)
    text = torch.randn(1, 16, CFG["text_dim"], generator=g).bfloat16().float()

    def latent(f_shift):
        x = torch.randn(1, CFG["in_channels"], 2, 8, 8, generator=g).bfloat16().float()
        return {"noisy_latents": x, "text_emb": text, "grid_id": ob.get_mesh_id(2, 4, 4, 0, f_shift=f_shift)[None],
                "timesteps": torch.rand(1, 2, generator=g) * 1000}

    def action(f_shift):
        x = torch.randn(1, CFG["action_dim"], 8, 4, 1, generator=g).bfloat16().float()
        return {"noisy_latents": x, "text_emb": text,
                "grid_id": ob.get_mesh_id(8, 4, 1, 0, f_shift=f_shift, action=True)[None],
                "timesteps": torch.rand(1, 8, generator=g) * 1000}

    calls = [(latent(0), 2, False), (latent(2), 2, False), (action(4), 0, True), (action(4), 1, True),
             ("clear", None, None), (action(4), 0, True)]
    for inp, update, action_mode in calls:
        if inp == "clear":
            for model in (m, rb_model, dev):
                for blk in model.blocks:
                    blk.attn1.clear_pred_cache("pos")
            continue
        with torch.no_grad():
            ref = m(inp, update_cache=update, action_mode=action_mode)
            rb = rb_model(_cuda(inp), update_cache=update, action_mode=action_mode)
            out = nm(_cuda(inp), update_cache=update, action_mode=action_mode)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        s = assert_parity(out, ref, rb, name=f"model KV lifecycle {'action' if action_mode else 'latent'} "
                                              f"update {update}")
        for bo, bn in zip(m.blocks, dev.blocks):
            co, cn = bo.attn1.attn_caches["pos"], bn.attn1.attn_caches["pos"]
            for k in ("id", "mask", "is_pred"):
                assert torch.equal(co[k], cn[k].cpu()), (update, k)
        print("kv lifecycle", "action" if action_mode else "latent", update, s)
