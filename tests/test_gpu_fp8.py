"""FP8-E4M3 path (no counterpart in the reference, which is bf16-only) against
the CPU model of the same scheme in oracle/fp8.py.

* wamb_quantize_rows: bit-exact against oracle.fp8.quant_rows (bytes and
  scales), bf16 and fp32 inputs, all-zero rows included.
* E4M3 GEMM (one-CTA and two-CTA kernels, all epilogues): against the fp32
  product of the dequantized operands; E4M3 x E4M3 products are exact in
  fp32, so the bound is the bf16 output rounding plus accumulation order
  (|ref| * 2^-8 + 1e-2), as for the bf16 GEMM.
* Block and 2-layer cfg2 stack in fp8 mode: against oracle.fp8.fp8_block.
  Tolerance: cosine >= 0.9995 and max |err| <= 0.1. The GPU quantizes values
  that differ from the fp32 model's in their last bits (bf16 operands of the
  attention, accumulation order), and such a value can land on the other
  side of an E4M3 rounding boundary (a step of 2^-3 relative): a few such
  flips per row move an output by a few 1e-3, far above bf16 noise, so the
  bf16 gate (cos 0.9999, 2e-2) does not apply.
* The same block and stack outputs against the unquantized fp32 oracle:
  cosine >= 0.999, the north-star's FP8 bound.
"""
import pytest
import torch

from blockutil import RESULTS, make_inputs, make_oracle_block, stats, to_device_block
from oracle import fp8 as of8
from oracle import wan_block as ob
from wam_ops import _lib, configs, ops
from wam_ops.native import NativeBlock
from wam_ops.stack import NativeStack

pytestmark = pytest.mark.gpu

COS_MIN_FP8 = 0.9995
MAX_ABS_FP8 = 0.1
COS_MIN_FP8_VS_FP32 = 0.999   # north_star: "FP8: cosine >= 0.999" against the fp32 reference


def _gate(out, ref, exact_ref=None, name=None):
    s = stats(out, ref)
    if exact_ref is not None:
        s["vs_unquantized"] = stats(out, exact_ref)
    if name is not None:
        RESULTS.append(dict(s, name=name, dtype="fp8"))
    assert s["finite"] and s["cos"] >= COS_MIN_FP8 and s["max_abs"] <= MAX_ABS_FP8, s
    if exact_ref is not None:
        assert s["vs_unquantized"]["cos"] >= COS_MIN_FP8_VS_FP32, s
    return s


@pytest.mark.parametrize("dtype,m,k", [(torch.bfloat16, 300, 3072), (torch.float32, 50, 1536),
                                       (torch.bfloat16, 7, 14336)])
def test_quantize_rows_bitwise(cuda_device, dtype, m, k):
    g = torch.Generator().manual_seed(m + k)
    x = (torch.randn(m, k, generator=g) * torch.logspace(-3, 3, m)[:, None]).to(dtype)
    x[1] = 0
    x[-1, 5] = 1e4
    q, s = ops.quantize_rows(x.cuda())
    torch.cuda.synchronize()
    qr, sr = of8.quant_rows(x)
    assert torch.equal(s.cpu(), sr)
    qb, rb = q.cpu().view(torch.uint8), qr.view(torch.uint8)
    diff = qb != rb
    # Only the sign of a zero may differ (an underflow to -0 vs +0); every
    # other byte is identical.
    assert torch.equal(q.cpu().float(), qr.float()), (
        diff.sum().item(), x[diff][:8].tolist(), qb[diff][:8].tolist(), rb[diff][:8].tolist())
    print("zero-sign mismatches:", diff.sum().item())


def _close(out, ref):
    err = (out.float() - ref).abs()
    bound = ref.abs() * 2.0 ** -8 + 1e-2
    assert torch.isfinite(out.float()).all()
    assert (err <= bound).all(), f"max err {err.max().item()}"


def _deq(q, s):
    return q.float() * s[:, None]


# The last two shapes leave SMs idle at any tile width and take the cluster
# split-K path.
@pytest.mark.parametrize("m,k,n,groups", [(200, 256, 384, 3), (129, 1536, 1536, 1), (1040, 512, 3072, 3),
                                          (4096, 3072, 3072, 1), (128, 14336, 3072, 1), (224, 8192, 1536, 3)])
def test_linear_e4m3(cuda_device, m, k, n, groups):
    g = torch.Generator(device="cuda").manual_seed(m + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(groups)]
    bs = [torch.randn(n, device="cuda", generator=g).bfloat16() for _ in range(groups)]
    a8, sa = ops.quantize_rows(a)
    w8s = [ops.quantize_rows(w) for w in ws]
    out = ops.linear(a8, [w for w, _ in w8s], bs, a_scale=sa, w_scales=[s for _, s in w8s])
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    wd = torch.cat([_deq(w, s) for w, s in w8s], 0)
    ref = _deq(a8, sa) @ wd.t() + torch.cat(bs).float()
    _close(out, ref)


@pytest.mark.parametrize("m", [300, 1300])
def test_linear_e4m3_epilogues(cuda_device, m):
    g = torch.Generator(device="cuda").manual_seed(m)
    B, Q, D, K = 2, m // 2, 4608, 768
    a = torch.randn(B * Q, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(D, K, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(D, device="cuda", generator=g).bfloat16()
    a8, sa = ops.quantize_rows(a)
    w8, sw = ops.quantize_rows(w)
    base = _deq(a8, sa) @ _deq(w8, sw).t() + b.float()
    out = ops.linear(a8, w8, b, epilogue=_lib.EPI_GELU, a_scale=sa, w_scales=sw)
    _close(out, torch.nn.functional.gelu(base, approximate="tanh"))
    res = torch.randn(B * Q, D, device="cuda", generator=g)
    table = torch.randn(6, D, device="cuda", generator=g)
    temb = torch.randn(B, 1, 6, D, device="cuda", generator=g)
    out = torch.empty(B * Q, D, device="cuda", dtype=torch.float32)
    ops.linear(a8, w8, b, epilogue=_lib.EPI_RES_GATE, res=res, table=table, temb=temb,
               rows_per_batch=Q, gate_index=2, out=out, a_scale=sa, w_scales=sw)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    gate = (table[2][None, None] + temb[:, :, 2]).expand(B, Q, D).reshape(B * Q, D)
    _close(out, res + base * gate)


def test_block_fp8_kv_pool(cuda_device):
    """Small block with a KV pool: update 2 then update 0, fp8 vs the fp8 model."""
    D, H, F, Q, C = 256, 2, 512, 48, 32
    blk = make_oracle_block(D, F, H, seed=11)
    pool = 3 * Q
    blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, 1)
    ref_blk = of8.fp8_block(blk)
    dev = to_device_block(blk)
    dev.attn1.init_kv_cache("pos", pool, H, 128, "cuda", torch.bfloat16, 1)
    nb = NativeBlock(dev, fp8=True)
    for step, upd in enumerate((2, 0)):
        x, ctx, temb, rope = make_inputs(1, Q, D, C, H, seed=100 + step)
        with torch.no_grad():
            ref = ref_blk(x, ctx, temb, rope, update_cache=upd)
            exact = blk(x, ctx, temb, rope, update_cache=upd)
            out = nb(x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), rope.cuda(),
                     update_cache=upd, out_dtype=torch.float32)
        assert _lib.device_status() == 0
        s = _gate(out, ref, exact, name=f"fp8 block D256 update {upd}")
        print("fp8 block update", upd, s)
        oc, dc = ref_blk.attn1.attn_caches["pos"], dev.attn1.attn_caches["pos"]
        for k in ("id", "mask", "is_pred"):
            assert torch.equal(oc[k], dc[k].cpu()), k


def test_stack_fp8_cfg2_two_layers(cuda_device):
    """cfg2 shape (D 3072, F 14336, 880-token chunk over a 4400-slot pool),
    2 layers, fp8 mode vs the fp8 model."""
    cfg = configs.PRESETS["cfg2"]
    Q = cfg.tokens
    pool, hist = cfg.pool_chunks * Q, cfg.history_chunks * Q
    oracle, dev = [], []
    g = torch.Generator().manual_seed(5)
    for i in range(2):
        b = make_oracle_block(cfg.dim, cfg.ffn, cfg.heads, seed=500 + i, randomize=False)
        b.attn1.init_kv_cache("pos", pool, cfg.heads, 128, "cpu", torch.float32, 1)
        c = b.attn1.attn_caches["pos"]
        c["k"].copy_(torch.randn(c["k"].shape, generator=g).bfloat16().float())
        c["v"].copy_(torch.randn(c["v"].shape, generator=g).bfloat16().float())
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist) // Q
        d = to_device_block(b)
        d.attn1.init_kv_cache("pos", pool, cfg.heads, 128, "cuda", torch.bfloat16, 1)
        for k in ("k", "v", "id", "mask", "is_pred"):
            d.attn1.attn_caches["pos"][k].copy_(c[k])
        oracle.append(b)
        dev.append(d)
    fp8_oracle = [of8.fp8_block(b) for b in oracle]
    x = torch.randn(1, Q, cfg.dim, generator=g).bfloat16().float()
    ctx = torch.randn(1, cfg.context, cfg.dim, generator=g).bfloat16().float()
    temb = configs.make_temb(cfg, 1, "cpu", g)
    rope = configs.chunk_rope(cfg, f_shift=4)
    with torch.no_grad():
        ref = ob.stack_forward(fp8_oracle, x, ctx, temb, rope)
        exact = ob.stack_forward(oracle, x, ctx, temb, rope)
        stack = NativeStack(dev, fp8=True)
        stack.prepare_context(ctx.cuda().bfloat16())
        out = stack(x.cuda().bfloat16(), None, temb.cuda(), rope.cuda())
    assert _lib.device_status() == 0
    s = _gate(out, ref, exact, name="fp8 cfg2 2 layers")
    print("fp8 cfg2 2-layer", s)


def test_block_fp8_large_m(cuda_device):
    """M = 1040 (the warp-per-row LayerNorm writes the E4M3 rows and scales)
    without a cache, fp8 vs the fp8 model and vs the fp32 block."""
    D, H, F, B, Q, C = 256, 2, 512, 2, 520, 48
    blk = make_oracle_block(D, F, H, seed=13)
    ref_blk = of8.fp8_block(blk)
    dev = to_device_block(blk)          # NativeBlock holds its block weakly
    nb = NativeBlock(dev, fp8=True)
    x, ctx, temb, rope = make_inputs(B, Q, D, C, H, seed=130)
    with torch.no_grad():
        ref = ref_blk(x, ctx, temb, rope)
        exact = blk(x, ctx, temb, rope)
        out = nb(x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), rope.cuda(), out_dtype=torch.float32)
    assert _lib.device_status() == 0
    s = _gate(out, ref, exact, name="fp8 block D256 M1040")
    print("fp8 block M1040", s)
