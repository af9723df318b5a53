"""Multi-layer parity and full-size properties of NativeStack (the 30-block
denoise step, model.py:1091-1098).

* 30 blocks of the configs[0] shape vs the fp32 oracle stack.
* configs[2] / configs[3] shapes (D 3072, 24 heads, FFN 14336, 3520-token
  history in a 4400-slot pool; 880-token chunk, or 4 candidates x 32 tokens
  with candidate_cache_rows = [0, 0, 0, 0]) on 2 layers vs the oracle (the
  fp32 oracle needs ~1 s per layer there).
* Full 30-layer configs[2] step: CUDA-graph replay equals the eager forward
  bit for bit, and repeated update_cache=0 steps leave the pool metadata
  unchanged (size-independent properties).

Gate (tests/blockutil.py): cosine >= 0.9999 and |err| <= 2e-2 against the
fp32 oracle for the stack's fp32 output (the residual stream the layers
pass each other), and 2e-2 plus half a bf16 ulp for its bf16 drop-in output.
Inputs follow the configs: weights N(0, 0.02), temb from the timestep chain.
"""
import pytest
import torch

from blockutil import assert_parity, make_oracle_block, to_device_block
from oracle import wan_block as ob
from wam_ops import _lib, configs
from wam_ops.stack import NativeStack

pytestmark = pytest.mark.gpu


def _oracle_stack(cfg, layers, seed):
    return [make_oracle_block(cfg.dim, cfg.ffn, cfg.heads, seed=seed + i, randomize=False)
            for i in range(layers)]


def _inputs(cfg, B, Q, seed, per_token=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, Q, cfg.dim, generator=g).bfloat16().float()
    ctx = torch.randn(B, cfg.context, cfg.dim, generator=g).bfloat16().float()
    temb = configs.make_temb(cfg, B, "cpu", g, per_token=per_token)
    return x, ctx, temb


def _f32(x):
    return torch.empty(x.shape, dtype=torch.float32, device="cuda")


def _run_reference_bf16(blocks, x, ctx, temb, rope, **kw):
    h = x.cuda().bfloat16()
    with torch.no_grad():
        for b in blocks:
            h = b(h, ctx.cuda().bfloat16(), temb.cuda(), rope.cuda(), **kw)
    return h


def test_cfg1_thirty_layers(cuda_device):
    cfg = configs.PRESETS["cfg1"]
    Q = cfg.tokens
    oracle = _oracle_stack(cfg, cfg.layers, seed=100)
    x, ctx, temb = _inputs(cfg, 1, Q, seed=1)
    rope = configs.chunk_rope(cfg)
    with torch.no_grad():
        ref = ob.stack_forward(oracle, x, ctx, temb, rope)
    dev_blocks = [to_device_block(b) for b in oracle]
    rb = _run_reference_bf16([to_device_block(b) for b in oracle], x, ctx, temb, rope)
    stack = NativeStack(dev_blocks)
    with torch.no_grad():
        stack.prepare_context(ctx.cuda().bfloat16())
        out32 = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda(), out=_f32(x))
        out = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda())
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    s32 = assert_parity(out32, ref, rb, name="cfg1 30 layers fp32-out")
    s = assert_parity(out, ref, rb, name="cfg1 30 layers bf16-out")
    print("cfg1 30-layer parity", s32, s)


def _pool_blocks(cfg, layers, seed, pool_batch):
    """Oracle blocks with a prefilled history (fp32 CPU) and bf16 GPU copies
    with the identical history."""
    Q = configs.PRESETS["cfg2"].tokens
    pool, hist = cfg.pool_chunks * Q, cfg.history_chunks * Q
    oracle = _oracle_stack(cfg, layers, seed)
    g = torch.Generator().manual_seed(seed)
    dev, tbf = [], []
    for b in oracle:
        b.attn1.init_kv_cache("pos", pool, cfg.heads, 128, "cpu", torch.float32, pool_batch)
        c = b.attn1.attn_caches["pos"]
        c["k"].copy_(torch.randn(c["k"].shape, generator=g).bfloat16().float())
        c["v"].copy_(torch.randn(c["v"].shape, generator=g).bfloat16().float())
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist) // Q
        for lst in (dev, tbf):
            d = to_device_block(b)
            d.attn1.init_kv_cache("pos", pool, cfg.heads, 128, "cuda", torch.bfloat16, pool_batch)
            dc = d.attn1.attn_caches["pos"]
            for k in ("k", "v"):
                dc[k].copy_(c[k])
            for k in ("id", "mask", "is_pred"):
                dc[k].copy_(c[k])
            lst.append(d)
    return oracle, dev, tbf


def test_cfg2_pool_path_two_layers(cuda_device):
    cfg = configs.PRESETS["cfg2"]
    oracle, dev, tbf = _pool_blocks(cfg, 2, seed=200, pool_batch=1)
    x, ctx, temb = _inputs(cfg, 1, cfg.tokens, seed=2)
    rope = configs.chunk_rope(cfg, f_shift=4)
    with torch.no_grad():
        ref = ob.stack_forward(oracle, x, ctx, temb, rope)
    rb = _run_reference_bf16(tbf, x, ctx, temb, rope)
    stack = NativeStack(dev)
    with torch.no_grad():
        stack.prepare_context(ctx.cuda().bfloat16())
        out32 = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda(), out=_f32(x))
        out = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda())
    assert _lib.device_status() == 0
    assert_parity(out32, ref, rb, name="cfg2 2 layers fp32-out")
    assert_parity(out, ref, rb, name="cfg2 2 layers bf16-out")
    for o, d in zip(oracle, dev):
        oc, dc = o.attn1.attn_caches["pos"], d.attn1.attn_caches["pos"]
        for k in ("id", "mask", "is_pred"):
            assert torch.equal(oc[k], dc[k].cpu()), k


def test_cfg3_candidates_two_layers(cuda_device):
    cfg = configs.PRESETS["cfg3"]
    oracle, dev, tbf = _pool_blocks(cfg, 2, seed=300, pool_batch=1)
    B, Q = cfg.candidates, cfg.tokens
    x, ctx, temb = _inputs(cfg, B, Q, seed=3, per_token=Q)
    rope = configs.chunk_rope(cfg, f_shift=4)
    rows = torch.zeros(B, dtype=torch.int64)
    with torch.no_grad():
        ref = ob.stack_forward(oracle, x, ctx, temb, rope, candidate_cache_rows=rows)
    rb = _run_reference_bf16(tbf, x, ctx, temb, rope, candidate_cache_rows=rows.cuda())
    stack = NativeStack(dev)
    with torch.no_grad():
        stack.prepare_context(ctx.cuda().bfloat16())
        out32 = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda(), candidate_cache_rows=rows.cuda(),
                      out=_f32(x))
        out = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda(), candidate_cache_rows=rows.cuda())
    assert _lib.device_status() == 0
    assert_parity(out32, ref, rb, name="cfg3 2 layers fp32-out")
    assert_parity(out, ref, rb, name="cfg3 2 layers bf16-out")


def test_cfg2_full_step_graph_properties(cuda_device):
    """30-layer configs[2] step: graph replay == eager (bitwise) and the KV
    metadata is unchanged by update_cache=0 steps."""
    cfg = configs.PRESETS["cfg2"]
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(7)
    blocks = configs.build_blocks(cfg, dev, seed=7)
    configs.fill_history(blocks, cfg, dev, gen, pool_batch=1)
    meta0 = [{k: b.attn1.attn_caches["pos"][k].clone() for k in ("id", "mask", "is_pred")} for b in blocks]
    stack = NativeStack(blocks)
    ctx = torch.randn(1, cfg.context, cfg.dim, generator=gen, device=dev).bfloat16()
    x = torch.randn(1, cfg.tokens, cfg.dim, generator=gen, device=dev).bfloat16()
    temb = configs.make_temb(cfg, 1, dev, gen)
    rope = configs.chunk_rope(cfg).to(dev)
    with torch.no_grad():
        stack.prepare_context(ctx)
        eager = stack(x, None, temb, rope).clone()
        stack.capture(x, None, temb, rope)
        replay1 = stack.replay().clone()
        replay2 = stack.replay(x, temb).clone()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert torch.isfinite(eager.float()).all()
    assert torch.equal(eager, replay1) and torch.equal(eager, replay2)
    for b, m in zip(blocks, meta0):
        c = b.attn1.attn_caches["pos"]
        assert torch.equal(c["mask"], m["mask"])
        new = (c["id"] != m["id"])
        # update 0 writes ids of the new (then hidden) slots only
        assert not (new & m["mask"]).any()
        assert torch.equal(c["is_pred"] & m["mask"], m["is_pred"] & m["mask"])
