"""Helpers shared by the block parity tests: seeded oracle blocks, their
bf16/fp32 GPU copies, the parity statistics and the stated tolerance.

Parity gate ("bf16: cosine >= 0.9999 and max abs error
<= 2e-2 vs an fp32 reference"), on the same bf16-representable weights and
inputs, element by element:

    cosine >= 0.9999  and  |out - ref| <= 2e-2 + r * ulp_bf16(|out|) / 2

r is the number of times the compared value itself was rounded to bf16 on
its way out: 0 for the fp32 outputs (the block's and the stack's fp32
residual-stream mode), 1 for a bf16 output (the drop-in block output, pool
K/V rows, cross K/V), k for a state re-rounded to bf16 after each of k
updates. The bf16 rounding of the output itself (half an ulp: 0.0156 at
|x| in [4, 8)) is the only allowance; nothing depends on the reference's own
bf16 error (E_ref), which is recorded beside each result for comparison.

Every checked result is appended to RESULTS; when WAMB_PARITY_OUT names a
file, conftest.py writes them there as JSON at the end of the session.
"""
import copy

import torch
import torch.nn.functional as F

from oracle import wan_block as ob

COS_MIN = 0.9999
MAX_ABS = 2e-2


def make_oracle_block(dim, ffn, heads, seed, cross_attn_norm=True, randomize=True):
    """fp32 CPU oracle block with bf16-representable weights (so that the
    comparison measures the kernels, not weight rounding)."""
    torch.manual_seed(seed)
    blk = ob.WanTransformerBlock(dim, ffn, heads, cross_attn_norm=cross_attn_norm, eps=1e-6)
    with torch.no_grad():
        for name, p in blk.named_parameters():
            if name.endswith("scale_shift_table"):
                p.copy_(torch.randn_like(p) / dim ** 0.5)
            elif "norm" in name and name.endswith("weight"):
                p.copy_(1.0 + 0.1 * torch.randn_like(p) if randomize else torch.ones_like(p))
            elif "norm" in name and name.endswith("bias"):
                p.copy_(0.1 * torch.randn_like(p) if randomize else torch.zeros_like(p))
            elif name.endswith("weight"):
                p.copy_(torch.randn_like(p) * 0.02)
            else:
                p.copy_(0.02 * torch.randn_like(p) if randomize else torch.zeros_like(p))
            p.copy_(p.bfloat16().float())
    return blk.eval()


def to_device_block(blk, device="cuda"):
    """GPU copy with the reference dtype policy: fp32 modulation table and
    norms (keep_in_fp32, model.py:812-825), bf16 everything else."""
    g = copy.deepcopy(blk)
    keep32 = ("scale_shift_table", "norm1", "norm2", "norm3")
    for name, p in g.named_parameters():
        fp32 = any(name.startswith(k) for k in keep32)
        p.data = p.data.to(device=device, dtype=torch.float32 if fp32 else torch.bfloat16).contiguous()
    g.attn1.attn_caches = {}
    return g


def stats(out, ref):
    out = out.float().cpu()
    ref = ref.float().cpu()
    err = (out - ref).abs()
    cos = F.cosine_similarity(out.double().flatten(), ref.double().flatten(), dim=0).item()
    return {"max_abs": err.max().item(), "cos": cos, "finite": bool(torch.isfinite(out).all())}


def half_ulp_bf16(x):
    """Half the spacing of bf16 numbers at |x| (a bound on the error of
    rounding a value to the bf16 number x)."""
    a = x.float().abs().clamp_min(2.0 ** -126)
    return torch.exp2(torch.floor(torch.log2(a)) - 8.0)


RESULTS = []


def assert_parity(out, ref, ref_bf16=None, cos_min=COS_MIN, max_abs=MAX_ABS, roundings=None, name=None):
    """The stated gate (module docstring). roundings defaults to 1 for a
    bf16 `out` and 0 otherwise; `ref_bf16` (optional) is the reference
    block's own bf16 output on the same inputs, recorded as E_ref only."""
    s = stats(out, ref)
    assert s["finite"], s
    if roundings is None:
        roundings = 1 if out.dtype == torch.bfloat16 else 0
    o = out.float().cpu()
    err = (o - ref.float().cpu()).abs()
    bound = max_abs + roundings * half_ulp_bf16(o)
    excess = (err - bound).max().item()
    s["roundings"] = roundings
    s["bound_at_max"] = bound.flatten()[err.flatten().argmax()].item()
    s["worst_margin"] = -excess
    if ref_bf16 is not None:
        s["E_ref"] = stats(ref_bf16, ref)["max_abs"]
    if name is not None:
        RESULTS.append(dict(s, name=name, dtype=str(out.dtype).replace("torch.", "")))
    assert s["cos"] >= cos_min and excess <= 0.0, s
    return s


def reference_bf16(dev_block, x, ctx, temb, rope, **kw):
    """The reference block (oracle module) executed in bf16 with torch ops on
    the GPU: the accuracy the reference itself reaches in bf16."""
    with torch.no_grad():
        return dev_block(x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(),
                         None if rope is None else rope.cuda(), **kw)


def make_inputs(B, Q, D, C, heads, seed, temb_len=1, temb_dtype=torch.float32, ctx_batch=None):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(B, Q, D, generator=g).bfloat16().float()
    ctx = torch.randn(ctx_batch or B, C, D, generator=g).bfloat16().float()
    temb = (torch.randn(B, temb_len, 6, D, generator=g) * 0.5).to(temb_dtype).float()
    grid = ob.get_mesh_id(max(1, Q // 8), 4, 2, 0)[:, :Q]
    if grid.shape[1] < Q:
        grid = torch.cat([grid, ob.get_mesh_id(1, Q - grid.shape[1], 1, 0, action=True)], 1)
    rope = ob.WanRotaryPosEmbed(128)(grid[None])[:, :, None]
    return x, ctx, temb, rope
