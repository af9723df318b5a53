"""tcgen05 GEMM (wamb_linear) against a torch fp32 reference on the GPU.

Shapes with M >= 512 and N per group a multiple of 256 take the two-CTA
(cta_group::2) kernel when they have at least 74 256 x 256 tiles, or when
the stream-K scratch lets them share a partly filled last round over all
SM pairs; residual-epilogue shapes with N per group a multiple of 192 take it with
256 x 192 tiles when the cost model rates that faster (the M 880, N 3072
projections);
the others take the one-CTA kernel with 64/128/192/256-column tiles, split
along K across a thread-block cluster when the tiles alone would leave SMs
idle.

Tolerance: the kernel accumulates in fp32 and rounds once to bf16, so the
error against an fp32 reference of the same bf16 operands is bounded by the
bf16 output rounding (|x| * 2^-8) plus fp32 accumulation-order noise.
"""
import pytest
import torch

from wam_ops import _lib, ops

pytestmark = pytest.mark.gpu


def _ref(a, ws, bs):
    w = torch.cat(ws, 0).float()
    y = a.float() @ w.t()
    if bs[0] is not None:
        y = y + torch.cat(bs, 0).float()
    return y


def _close(out, ref):
    err = (out.float() - ref).abs()
    bound = ref.abs() * 2.0 ** -8 + 1e-2
    assert torch.isfinite(out.float()).all()
    assert (err <= bound).all(), f"max err {err.max().item()} / worst ratio {(err / bound).max().item()}"


@pytest.mark.parametrize("m,k,n,groups", [
    (128, 64, 64, 1), (200, 256, 256, 1), (880, 512, 384, 3), (1592, 1536, 1536, 1),
    (64, 3072, 1024, 1), (7, 128, 128, 2),
    # two-CTA path: M tail whose second 128-row half is wholly out of range
    (1040, 512, 3072, 3), (4096, 3072, 3072, 1),
])
def test_linear_bias(cuda_device, m, k, n, groups):
    g = torch.Generator(device="cuda").manual_seed(m * 7 + k)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(groups)]
    bs = [torch.randn(n, device="cuda", generator=g).bfloat16() for _ in range(groups)]
    out = ops.linear(a, ws, bs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    _close(out, _ref(a, ws, bs))


def test_linear_gelu(cuda_device):
    g = torch.Generator(device="cuda").manual_seed(1)
    a = torch.randn(300, 256, device="cuda", generator=g).bfloat16()
    w = (torch.randn(512, 256, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(512, device="cuda", generator=g).bfloat16()
    out = ops.linear(a, w, b, epilogue=_lib.EPI_GELU)
    ref = torch.nn.functional.gelu(_ref(a, [w], [b]), approximate="tanh")
    _close(out, ref)


@pytest.mark.parametrize("temb_len,temb_f32", [(1, True), (40, False)])
def test_linear_residual_gate(cuda_device, temb_len, temb_f32):
    g = torch.Generator(device="cuda").manual_seed(2)
    B, Q, D, K = 3, 40, 256, 512
    a = torch.randn(B * Q, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(D, K, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(D, device="cuda", generator=g).bfloat16()
    res = torch.randn(B * Q, D, device="cuda", generator=g).bfloat16()
    table = torch.randn(6, D, device="cuda", generator=g)
    temb = torch.randn(B, temb_len, 6, D, device="cuda", generator=g)
    if not temb_f32:
        temb = temb.bfloat16()
    out = ops.linear(a, w, b, epilogue=_lib.EPI_RES_GATE, res=res, table=table, temb=temb,
                     rows_per_batch=Q, gate_index=2)
    gate = (table[2][None, None] + temb[:, :, 2].float()).expand(B, Q, D).reshape(B * Q, D)
    ref = res.float() + _ref(a, [w], [b]) * gate
    _close(out, ref)
    out2 = ops.linear(a, w, b, epilogue=_lib.EPI_RES, res=res)
    _close(out2, res.float() + _ref(a, [w], [b]))


@pytest.mark.parametrize("res_f32,per_token", [(False, False), (True, False), (True, True)])
def test_linear_pair_epilogues(cuda_device, res_f32, per_token):
    """Two-CTA kernel (M 1300, N 4608): GELU, and the gated residual with a
    bf16 or fp32 residual stream and fp32 output; the gate's modulation row
    per batch row (650 rows each, so one warp straddles two batch rows) or
    per token (bf16)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    B, Q, D, K = 2, 650, 4608, 768
    a = torch.randn(B * Q, K, device="cuda", generator=g).bfloat16()
    w = (torch.randn(D, K, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(D, device="cuda", generator=g).bfloat16()
    out = ops.linear(a, w, b, epilogue=_lib.EPI_GELU)
    _close(out, torch.nn.functional.gelu(_ref(a, [w], [b]), approximate="tanh"))
    res = torch.randn(B * Q, D, device="cuda", generator=g)
    if not res_f32:
        res = res.bfloat16()
    table = torch.randn(6, D, device="cuda", generator=g)
    temb = torch.randn(B, Q if per_token else 1, 6, D, device="cuda", generator=g)
    if per_token:
        temb = temb.bfloat16()
    out = torch.empty(B * Q, D, device="cuda", dtype=torch.float32)
    ops.linear(a, w, b, epilogue=_lib.EPI_RES_GATE, res=res, table=table, temb=temb,
               rows_per_batch=Q, gate_index=5, out=out)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    gate = (table[5][None, None] + temb[:, :, 5].float()).expand(B, Q, D).reshape(B * Q, D)
    _close(out, res.float() + _ref(a, [w], [b]) * gate)


@pytest.mark.parametrize("m,k,n,groups,epi", [
    (128, 8192, 3072, 1, "bias"), (128, 14336, 3072, 1, "res_gate"), (224, 8192, 1536, 3, "bias"),
    (100, 4096, 2560, 1, "gelu"), (128, 14336, 3072, 1, "res"),
    # K 3072: the verify batch's O / cross projections and a 2 x 128-row tile column
    (128, 3072, 3072, 1, "res_bf16"), (224, 3072, 3072, 1, "res_gate"), (256, 3072, 3072, 3, "bias"),
])
def test_linear_split_k(cuda_device, m, k, n, groups, epi):
    """Small M (the output tiles leave SMs idle): K is split across the CTAs
    of a thread-block cluster, which sum their partials in split order
    through shared memory; the result meets the unsplit GEMM's bound and is
    bitwise the same on a second call."""
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.02).bfloat16() for _ in range(groups)]
    bs = [torch.randn(n, device="cuda", generator=g).bfloat16() for _ in range(groups)]
    N = n * groups
    kw, ref = {}, _ref(a, ws, bs)
    if epi == "gelu":
        kw["epilogue"] = _lib.EPI_GELU
        ref = torch.nn.functional.gelu(ref, approximate="tanh")
    elif epi == "res_bf16":
        res = torch.randn(m, N, device="cuda", generator=g).bfloat16()
        kw.update(epilogue=_lib.EPI_RES, res=res)
        ref = res.float() + ref
    elif epi in ("res", "res_gate"):
        res = torch.randn(m, N, device="cuda", generator=g)
        kw.update(epilogue=_lib.EPI_RES if epi == "res" else _lib.EPI_RES_GATE, res=res)
        if epi == "res_gate":
            table = torch.randn(6, N, device="cuda", generator=g)
            temb = torch.randn(1, 1, 6, N, device="cuda", generator=g)
            kw.update(table=table, temb=temb, rows_per_batch=m, gate_index=5)
            ref = res + ref * (table[5] + temb[0, 0, 5])[None]
        else:
            ref = res + ref
        kw["out"] = torch.empty(m, N, device="cuda", dtype=torch.float32)
    out1 = ops.linear(a, ws, bs, **kw)
    out1 = out1.clone()
    out2 = ops.linear(a, ws, bs, **kw)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    _close(out1, ref)
    assert torch.equal(out1, out2)            # deterministic: partials summed in split order


# ------------------------------------------------------------------ stream-K
# M >= 512 with a stream-K scratch (ops.linear passes one): when the
# 256 x 256 tiles leave the last round over the SM pairs partly filled, the
# two-CTA kernel shares that round's tiles x k-blocks evenly over every
# pair, and a tile split between pairs is finished from the others' fp32
# partials.
def _sk_flags_zero(dev):
    ws = ops.sk_workspace(dev)
    return bool((ws[:8192] == 0).all())


@pytest.mark.parametrize("m,k,n,groups", [
    (880, 14336, 3072, 1),     # FFN2 shape: 48 tiles over 74 pairs, 224 k-blocks each
    (880, 8192, 3072, 3),      # three weight groups: one full round + 70 shared tiles
    (2000, 8960, 1536, 1),     # D 1536 FFN2 shape, ragged last row block
    (7040, 14336, 3072, 1),    # 336 tiles: 4 full rounds + 40 shared tiles
    (880, 3072, 3072, 1),      # K 3072: no stream-K (the one-CTA path)
    (512, 8192, 256, 1),       # too few tiles to share: no stream-K
])
def test_linear_stream_k(cuda_device, m, k, n, groups):
    g = torch.Generator(device="cuda").manual_seed(m + k + n)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    ws = [(torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16() for _ in range(groups)]
    bs = [torch.randn(n, device="cuda", generator=g).bfloat16() for _ in range(groups)]
    out = ops.linear(a, ws, bs)
    again = ops.linear(a, ws, bs)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert _sk_flags_zero(a.device)
    _close(out, _ref(a, ws, bs))
    assert torch.equal(out, again)   # fixed summation order: no dependence on timing


def test_linear_stream_k_epilogues(cuda_device):
    """Gated fp32 residual (the FFN output projection at M 880) and GELU
    through the stream-K path, against the fp32 reference."""
    m, k, n, B = 880, 14336, 3072, 2
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.01).bfloat16()
    b = torch.randn(n, device="cuda", generator=g).bfloat16()
    res = torch.randn(m, n, device="cuda", generator=g)
    table = torch.randn(6, n, device="cuda", generator=g) * 0.1
    temb = torch.randn(B, 1, 6, n, device="cuda", generator=g) * 0.1
    out = torch.empty(m, n, device="cuda")
    ops.linear(a, w, b, epilogue=_lib.EPI_RES_GATE, res=res, table=table, temb=temb, rows_per_batch=m // B,
               gate_index=2, out=out)
    gelu = ops.linear(a, w, b, epilogue=_lib.EPI_GELU)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert _sk_flags_zero(a.device)
    base = _ref(a, [w], [b])
    gate = (table[2][None, None] + temb[:, :, 2]).expand(B, m // B, n).reshape(m, n)
    err = (out - (res + base * gate)).abs().max().item()
    assert err <= 5e-3, err
    _close(gelu, torch.nn.functional.gelu(base, approximate="tanh"))


def test_linear_stream_k_fp8(cuda_device):
    m, k, n = 880, 16384, 3072     # 128 E4M3 k-blocks
    g = torch.Generator(device="cuda").manual_seed(6)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(n, device="cuda", generator=g).bfloat16()
    a8, sa = ops.quantize_rows(a)
    w8, sw = ops.quantize_rows(w)
    out = ops.linear(a8, w8, b, a_scale=sa, w_scales=sw)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    assert _sk_flags_zero(a.device)
    deq = lambda q, s: q.float() * s[:, None]  # noqa: E731
    _close(out, deq(a8, sa) @ deq(w8, sw).t() + b.float())



@pytest.mark.parametrize("m,k,n", [
    (880, 3072, 3072),     # O / cross-O projections of one cfg2 chunk: 64 pair tiles of 256 x 192
    (1592, 1536, 1536),    # D 1536 projections: the last pair tile's second half out of range
    (600, 1536, 3072),     # 3 x 16 pair tiles, a ragged last row block
])
def test_linear_pair192(cuda_device, m, k, n):
    """Two-CTA kernel with 256 x 192 tiles (three 32-column chunks per
    epilogue warp; the residual epilogues of N % 192 == 0 shapes with too
    few 256 x 256 tiles): the gated fp32 residual with fp32 output and the
    plain bf16 residual, bitwise repeatable."""
    g = torch.Generator(device="cuda").manual_seed(m + 3 * k + n)
    B = 2
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.03).bfloat16()
    b = torch.randn(n, device="cuda", generator=g).bfloat16()
    res = torch.randn(m, n, device="cuda", generator=g)
    table = torch.randn(6, n, device="cuda", generator=g) * 0.1
    temb = torch.randn(B, 1, 6, n, device="cuda", generator=g) * 0.1
    o32, again = torch.empty(m, n, device="cuda"), torch.empty(m, n, device="cuda")
    for o in (o32, again):
        ops.linear(a, w, b, epilogue=_lib.EPI_RES_GATE, res=res, table=table, temb=temb,
                   rows_per_batch=m // B, gate_index=2, out=o)
    res16 = res.bfloat16()
    o16 = ops.linear(a, w, b, epilogue=_lib.EPI_RES, res=res16)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    base = _ref(a, [w], [b])
    gate = (table[2][None, None] + temb[:, :, 2]).expand(B, m // B, n).reshape(m, n)
    err = (o32 - (res + base * gate)).abs().max().item()
    assert err <= 5e-3, err
    assert torch.equal(o32, again)
    _close(o16, res16.float() + base)


def test_linear_pair192_fp8(cuda_device):
    """E4M3 operands through the 256 x 192 pair tiles (fp32 residual)."""
    m, k, n = 880, 3072, 3072
    g = torch.Generator(device="cuda").manual_seed(8)
    a = torch.randn(m, k, device="cuda", generator=g).bfloat16()
    w = (torch.randn(n, k, device="cuda", generator=g) * 0.05).bfloat16()
    b = torch.randn(n, device="cuda", generator=g).bfloat16()
    res = torch.randn(m, n, device="cuda", generator=g)
    a8, sa = ops.quantize_rows(a)
    w8, sw = ops.quantize_rows(w)
    out = torch.empty(m, n, device="cuda")
    ops.linear(a8, w8, b, a_scale=sa, w_scales=sw, epilogue=_lib.EPI_RES, res=res, out=out)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    deq = lambda q, s: q.float() * s[:, None]  # noqa: E731
    err = (out - (res + deq(a8, sa) @ deq(w8, sw).t() + b.float())).abs().max().item()
    assert err <= 5e-3, err

