"""Block parity: the B200 native block (through install_block / NativeBlock,
i.e. through the C ABI) against the fp32 CPU oracle restatement of
WanTransformerBlock.forward (model.py:741-794), including the KV-cache
lifecycle (update_cache 0/1/2, id eviction), candidate verification and the
prepared cross-K/V variant.

Tolerance (tests/blockutil.py): cosine >= 0.9999 and
|err| <= 2e-2 against the fp32 oracle on identical bf16-representable
weights and inputs, plus half a bf16 ulp of the value for outputs stored in
bf16 (the drop-in output, pool K/V rows, cross K/V). The block's fp32 output
mode gets no allowance. Cache metadata (id, mask, is_pred) must match
exactly. The small cases use a stress modulation (temb ~ 0.5 N(0,1): scales
and gates up to +-2); configs[0] uses its own temb chain.
"""
import pytest
import torch

from blockutil import (assert_parity, make_inputs, make_oracle_block, reference_bf16, stats,
                       to_device_block)
from wam_ops import _lib, configs
from wam_ops.install import install_block, install_model
from wam_ops.whole_layer import WholeLayerBlock

pytestmark = pytest.mark.gpu


def _run_native(g, x, ctx, temb, rope, temb_dtype=torch.float32, out_dtype=torch.float32, **kw):
    """Through install_block; out_dtype=float32 reads the block's fp32 output
    mode (NativeBlock(out_dtype=...)), bfloat16 the plain drop-in call."""
    with torch.no_grad(), install_block(g):
        args = (x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda().to(temb_dtype),
                None if rope is None else rope.cuda())
        if out_dtype == torch.bfloat16:
            out = g(*args, **kw)
        else:
            native = g._native_block
            out = native(*args, kw.pop("update_cache", 0), "pos", kw.pop("candidate_cache_rows", None),
                         out_dtype=out_dtype)
    assert _lib.device_status() == 0
    return out


@pytest.mark.parametrize("B,Q,C,temb_len,temb_dtype,rope,norm2", [
    (1, 40, 24, 1, torch.float32, True, True),
    (2, 130, 77, 130, torch.bfloat16, True, True),
    (3, 16, 512, 1, torch.float32, False, False),
    # M >= 1024: the warp-per-row LayerNorm (per-token bf16 modulation; Identity norm2)
    (2, 520, 64, 520, torch.bfloat16, True, True),
    (4, 260, 32, 1, torch.float32, False, False),
])
def test_block_no_cache(cuda_device, B, Q, C, temb_len, temb_dtype, rope, norm2):
    D, H, F = 256, 2, 512
    blk = make_oracle_block(D, F, H, seed=B * 10 + Q, cross_attn_norm=norm2)
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=Q, temb_len=temb_len, temb_dtype=temb_dtype)
    r = r if rope else None
    with torch.no_grad():
        ref = blk(x, ctx, temb, r)
    g = to_device_block(blk)
    rb = reference_bf16(to_device_block(blk), x, ctx, temb.to(temb_dtype).float(), r)
    tag = f"block D256 B{B} Q{Q} C{C} temb_len {temb_len}"
    assert_parity(_run_native(g, x, ctx, temb, r, temb_dtype), ref, rb, name=tag + " fp32-out")
    out = _run_native(g, x, ctx, temb, r, temb_dtype, out_dtype=torch.bfloat16)
    assert out.dtype == torch.bfloat16
    assert_parity(out, ref, rb, name=tag + " bf16-out")


def test_block_context_broadcast(cuda_device):
    D, H, F, B, Q, C = 256, 2, 512, 3, 24, 40
    blk = make_oracle_block(D, F, H, seed=3)
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=4, ctx_batch=1)
    with torch.no_grad():
        ref = blk(x, ctx.expand(B, -1, -1), temb, r)
    rb = reference_bf16(to_device_block(blk), x, ctx.expand(B, -1, -1), temb, r)
    assert_parity(_run_native(to_device_block(blk), x, ctx, temb, r), ref, rb, name="block context broadcast")


def _cache_equal(oc, gc, tc):
    """Metadata exactly; pool rows (bf16 by the cache schema) under the parity
    gate, bounded by the reference's own bf16 cache (tc) error."""
    assert torch.equal(oc["id"], gc["id"].cpu())
    assert torch.equal(oc["mask"], gc["mask"].cpu())
    assert torch.equal(oc["is_pred"], gc["is_pred"].cpu())
    valid = oc["mask"] | (oc["id"] >= 0)
    idx = valid.nonzero().squeeze(-1)
    for name in ("k", "v"):
        assert_parity(gc[name][:, idx.cuda()], oc[name][:, idx], tc[name][:, idx.cuda()])


@pytest.mark.parametrize("Q,pool", [
    (40, 100),
    (520, 1300),   # M 1040: the warp-per-row LayerNorm and RMS, K/V written into pool slots
])
def test_block_kv_lifecycle_and_eviction(cuda_device, Q, pool):
    """prefill (update 2) x2, denoise (update 0), commit prediction (update 1)
    with eviction of the oldest chunk, then denoise again."""
    D, H, F, B, C = 256, 2, 512, 2, 24
    blk = make_oracle_block(D, F, H, seed=11)
    g = to_device_block(blk)
    tb = to_device_block(blk)
    blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, B)
    g.attn1.init_kv_cache("pos", pool, H, 128, "cuda", torch.bfloat16, B)
    tb.attn1.init_kv_cache("pos", pool, H, 128, "cuda", torch.bfloat16, B)
    for step, update in enumerate((2, 2, 0, 1, 0)):
        x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=100 + step)
        with torch.no_grad():
            ref = blk(x, ctx, temb, r, update_cache=update)
        rb = reference_bf16(tb, x, ctx, temb, r, update_cache=update)
        out = _run_native(g, x, ctx, temb, r, update_cache=update)
        assert_parity(out, ref, rb, name=f"block KV lifecycle call {step} update {update}")
        _cache_equal(blk.attn1.attn_caches["pos"], g.attn1.attn_caches["pos"], tb.attn1.attn_caches["pos"])


@pytest.mark.parametrize("rows,Q", [
    ([0, 1, 1, 0], 16),           # different history rows: one CTA set per candidate
    ([1, 1, 1, 1], 16),           # one shared row: grouped candidates, split key tiles
    ([0] * 10, 16),               # grouped, 160 query rows: two tiles, private keys in two tiles
    ([0, 0, 0], 40),              # grouped, candidate boundaries inside a tile
])
def test_block_candidate_verification(cuda_device, rows, Q):
    D, H, F, Bp, C, pool = 256, 2, 512, 2, 24, 200
    blk = make_oracle_block(D, F, H, seed=21)
    g = to_device_block(blk)
    tb = to_device_block(blk)
    blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, Bp)
    g.attn1.init_kv_cache("pos", pool, H, 128, "cuda", torch.bfloat16, Bp)
    tb.attn1.init_kv_cache("pos", pool, H, 128, "cuda", torch.bfloat16, Bp)
    for step in range(2):
        x, ctx, temb, r = make_inputs(Bp, 70, D, C, H, seed=200 + step)
        with torch.no_grad():
            blk(x, ctx, temb, r, update_cache=2)
        reference_bf16(tb, x, ctx, temb, r, update_cache=2)
        _run_native(g, x, ctx, temb, r, update_cache=2)
    rows = torch.tensor(rows, dtype=torch.int64)
    B = len(rows)
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=300 + Q + B, temb_len=Q)
    before = {k: v.clone() for k, v in g.attn1.attn_caches["pos"].items()}
    with torch.no_grad():
        ref = blk(x, ctx, temb, r, candidate_cache_rows=rows)
    rb = reference_bf16(tb, x, ctx, temb, r, candidate_cache_rows=rows.cuda())
    out = _run_native(g, x, ctx, temb, r, candidate_cache_rows=rows.cuda())
    assert_parity(out, ref, rb, name=f"block candidates rows {rows.tolist()} Q{Q}")
    for k, v in g.attn1.attn_caches["pos"].items():
        # bitwise (an uninitialised pool may hold NaN patterns)
        assert torch.equal(v.view(torch.uint8), before[k].view(torch.uint8)), f"candidate path wrote the cache ({k})"


def test_block_rejects_bad_candidate_rows(cuda_device):
    D, H, F = 256, 2, 512
    blk = make_oracle_block(D, F, H, seed=31)
    g = to_device_block(blk)
    x, ctx, temb, r = make_inputs(2, 16, D, 8, H, seed=31)
    with pytest.raises(ValueError):
        _run_native(g, x, ctx, temb, r, candidate_cache_rows=torch.zeros(2, dtype=torch.int64, device="cuda"))


def test_whole_layer_prepared_context(cuda_device):
    D, H, F, B, Q, C = 256, 2, 512, 4, 32, 48
    blk = make_oracle_block(D, F, H, seed=41)
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=41)
    ctx[2] = ctx[0]
    ctx[3] = ctx[1]
    with torch.no_grad():
        ref = blk(x, ctx, temb, r)
    rb = reference_bf16(to_device_block(blk), x, ctx, temb, r)
    g = to_device_block(blk)
    with torch.no_grad():
        w = WholeLayerBlock(g)
        w.prepare_context(ctx.cuda().bfloat16(), precompute=True)
        assert w.context_roots is not None and w.context_roots.numel() == 2
        out = w(x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), r.cuda())
        dbg = w(x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), r.cuda(), debug=True)
    assert_parity(out, ref, rb, name="whole layer prepared context")
    assert torch.equal(dbg["output"], out)
    assert "modulated1" in dbg and "gelu" in dbg


@pytest.mark.parametrize("D,C,Bc", [(3072, 512, 1), (1536, 512, 2), (3072, 200, 3)])
def test_cross_kv_construction(cuda_device, D, C, Bc):
    """wamb_cross_kv (the prepared cross K/V: RMS(ctx W_k^T + b_k) * gamma_k
    and ctx W_v^T + b_v, model.py:612-615) against the oracle module's own
    to_k / norm_k / to_v in fp32: the per-chunk rebuild of one 512-token
    context at D 3072, two contexts at D 1536, and a ragged token count."""
    H = D // 128
    blk = make_oracle_block(D, 256, H, seed=53)
    ctx = torch.randn(Bc, C, D, generator=torch.Generator().manual_seed(53)).bfloat16().float()
    at = blk.attn2
    with torch.no_grad():
        k_ref, v_ref = at.norm_k(at.to_k(ctx)), at.to_v(ctx)
        g = to_device_block(blk)
        k_bf, v_bf = g.attn2.norm_k(g.attn2.to_k(ctx.cuda().bfloat16())), g.attn2.to_v(ctx.cuda().bfloat16())
        w = WholeLayerBlock(g)
        w.prepare_context(ctx.cuda().bfloat16(), precompute=True)
    k, v = w.context_kv
    assert k.shape == (Bc, C, D) and v.shape == (Bc, C, D)
    assert_parity(k, k_ref, k_bf, name=f"cross K D{D} C{C} Bc{Bc}")
    assert_parity(v, v_ref, v_bf, name=f"cross V D{D} C{C} Bc{Bc}")


def test_cfg0_single_block(cuda_device):
    """D 1536, 12 heads, FFN 8960, 1560 video (2 x 30 x 26) + 32
    action tokens, 512 context tokens, weights N(0, 0.02), biases 0, temb
    from t ~ U[0, 1000) through the sinusoidal Linear-SiLU-Linear chain,
    RoPE from the chunk's grid ids; against the fp32 oracle in both output
    modes."""
    cfg = configs.PRESETS["cfg0"]
    D, H, F, B, Q, C = cfg.dim, cfg.heads, cfg.ffn, 1, cfg.tokens, cfg.context
    blk = make_oracle_block(D, F, H, seed=0, randomize=False)
    g0 = torch.Generator().manual_seed(0)
    x = torch.randn(B, Q, D, generator=g0).bfloat16().float()
    ctx = torch.randn(B, C, D, generator=g0).bfloat16().float()
    temb = configs.make_temb(cfg, B, "cpu", g0)
    r = configs.chunk_rope(cfg)
    with torch.no_grad():
        ref = blk(x, ctx, temb, r)
    g = to_device_block(blk)
    rb = reference_bf16(to_device_block(blk), x, ctx, temb, r)
    s32 = assert_parity(_run_native(g, x, ctx, temb, r), ref, rb, name="cfg0 fp32-out")
    s16 = assert_parity(_run_native(g, x, ctx, temb, r, out_dtype=torch.bfloat16), ref, rb,
                        name="cfg0 bf16-out")
    print("cfg0 parity fp32-out", s32, "bf16-out", s16)


# Bound of the stress case below: with gates and scales up to +-2 the bf16
# operands of the two FFN GEMMs alone cost ~0.02 at this shape. A CPU model
# of the block that rounds every tensor-core operand to bf16 and computes
# everything else in fp32 (the floor of any bf16-operand datapath) is
# 0.0206 from the fp32 oracle here; rounding only the LN3 output gives
# 0.0158, only the GELU output 0.0148, every other operand alone < 0.004.
STRESS_MAX_ABS = 3e-2


def test_cfg0_shape_stress_modulation(cuda_device):
    """The configs[0] shape with the small cases' stress modulation (temb ~
    0.5 N(0,1), 14x the configs' temb): outside the configs' distribution,
    so the bound is the bf16-operand floor above plus margin, not 2e-2."""
    D, H, F, B, Q, C = 1536, 12, 8960, 1, 1592, 512
    blk = make_oracle_block(D, F, H, seed=0, randomize=False)
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=0)
    with torch.no_grad():
        ref = blk(x, ctx, temb, r)
    g = to_device_block(blk)
    rb = reference_bf16(to_device_block(blk), x, ctx, temb, r)
    s = assert_parity(_run_native(g, x, ctx, temb, r), ref, rb, max_abs=STRESS_MAX_ABS,
                      name="cfg0 shape, stress temb, fp32-out")
    print("cfg0-shape stress parity", s)


def test_install_model_restores_classes(cuda_device):
    D, H, F = 256, 2, 512

    class Model(torch.nn.Module):
        def __init__(self):
            super().__init__()
            self.blocks = torch.nn.ModuleList([to_device_block(make_oracle_block(D, F, H, seed=s))
                                               for s in range(2)])

    m = Model()
    kinds = [type(b) for b in m.blocks]
    with install_model(m, "optimized", execution_mode="persistent"):
        assert all(type(b).__name__ == "TransformerBlock" for b in m.blocks)
    assert [type(b) for b in m.blocks] == kinds
    assert all("_native_block" not in b.__dict__ for b in m.blocks)
