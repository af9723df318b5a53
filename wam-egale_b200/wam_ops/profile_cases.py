"""Small single-kernel cases for ncu captures (inputs larger than L2, a few
hundred MB on the device, 3 warm-up launches then `--launches` more).

  python wam-egale_b200/wam_ops/profile_cases.py ffn1 [--m 2048] [--launches 1] [--fp8]
  python wam-egale_b200/wam_ops/profile_cases.py attention [--q 880] [--pool 4400] [--batch 8]
  python wam-egale_b200/wam_ops/profile_cases.py rms | ln
  python wam-egale_b200/wam_ops/profile_cases.py small [--m 128] [--n 3072] [--k 14336]
  python wam-egale_b200/wam_ops/profile_cases.py verify_attention
  python wam-egale_b200/wam_ops/profile_cases.py res_gate [--m 4096] [--launches 1]

ffn1       FFN1 GEMM + GELU epilogue, M x 14336 x 3072 (cfg2 weights); --fp8: E4M3
           operands (quantized once before the timed launches)
attention  self attention of `batch` cfg2 rollouts over 4400-key pools (24 heads)
rms        RMSNorm + RoPE of the q/k/v projection output, K/V into the pool
ln         LayerNorm + adaLN modulation
verify_attention  cfg3 self attention: 4 candidates x 32 queries sharing one
           3520-slot history row of a 4400-slot pool (grouped candidates) plus
           their own keys, 24 heads
res_gate   the block's O projection: M x 3072 x 3072 GEMM with the gated fp32
           residual epilogue (out fp32 = res + gate * (acc + bias)), per-row
           modulation of 8 batch rows; prints its CUDA-event time next to the
           same GEMM with an ungated residual, a bias epilogue with fp32
           output and one with bf16 output
small      small-M GEMM + residual epilogue (the verify batch's O / FFN-out
           projections; cluster split-K where the tiles leave SMs idle); 12
           weight copies rotate so every launch streams its weights from HBM
"""
import argparse
import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parents[1]))

import torch  # noqa: E402

from wam_ops import _lib, configs, ops  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("case", choices=["ffn1", "attention", "rms", "ln", "small", "verify_attention", "res_gate"])
    ap.add_argument("--m", type=int, default=2048)
    ap.add_argument("--n", type=int, default=3072)
    ap.add_argument("--k", type=int, default=14336)
    ap.add_argument("--q", type=int, default=880)
    ap.add_argument("--pool", type=int, default=4400)
    ap.add_argument("--batch", type=int, default=8)
    ap.add_argument("--launches", type=int, default=1)
    ap.add_argument("--fp8", action="store_true")
    a = ap.parse_args()
    torch.set_grad_enabled(False)
    dev = torch.device("cuda", 0)
    g = torch.Generator(device=dev).manual_seed(0)
    D, H, F = 3072, 24, 14336
    if a.case == "ffn1":
        x = torch.randn(a.m, D, generator=g, device=dev).bfloat16()
        w = (torch.randn(F, D, generator=g, device=dev) * 0.02).bfloat16()
        b = torch.zeros(F, device=dev, dtype=torch.bfloat16)
        out = torch.empty(a.m, F, device=dev, dtype=torch.bfloat16)
        if a.fp8:
            x8, sx = ops.quantize_rows(x)
            w8, sw = ops.quantize_rows(w)
            run = lambda: ops.linear(x8, w8, b, epilogue=_lib.EPI_GELU, out=out,  # noqa: E731
                                     a_scale=sx, w_scales=sw)
        else:
            run = lambda: ops.linear(x, w, b, epilogue=_lib.EPI_GELU, out=out)  # noqa: E731
    elif a.case == "small":
        x = torch.randn(a.m, a.k, generator=g, device=dev).bfloat16()
        ws = [(torch.randn(a.n, a.k, generator=g, device=dev) * 0.02).bfloat16() for _ in range(12)]
        b = torch.zeros(a.n, device=dev, dtype=torch.bfloat16)
        res = torch.randn(a.m, a.n, generator=g, device=dev).bfloat16()
        out = torch.empty(a.m, a.n, device=dev, dtype=torch.bfloat16)
        it = iter(range(1 << 30))
        run = lambda: ops.linear(x, ws[next(it) % 12], b, epilogue=_lib.EPI_RES, out=out,  # noqa: E731
                                 res=res)
    elif a.case == "res_gate":
        cfg = configs.PRESETS["cfg2"]
        x = torch.randn(a.m, D, generator=g, device=dev).bfloat16()
        w = (torch.randn(D, D, generator=g, device=dev) * 0.02).bfloat16()
        b = torch.zeros(D, device=dev, dtype=torch.bfloat16)
        res = torch.randn(a.m, D, generator=g, device=dev)
        out = torch.empty(a.m, D, device=dev)
        out_bf = torch.empty(a.m, D, device=dev, dtype=torch.bfloat16)
        table = torch.randn(6, D, generator=g, device=dev) / D ** 0.5
        temb = configs.make_temb(cfg, 8, dev, g)
        gate = dict(table=table, temb=temb, rows_per_batch=a.m // 8, gate_index=2)
        run = lambda: ops.linear(x, w, b, epilogue=_lib.EPI_RES_GATE, out=out, res=res, **gate)  # noqa: E731
        variants = (("res_gate", run),
                    ("res_f32", lambda: ops.linear(x, w, b, epilogue=_lib.EPI_RES, out=out, res=res)),
                    ("bias_f32", lambda: ops.linear(x, w, b, out=out)),
                    ("bias_bf16", lambda: ops.linear(x, w, b, out=out_bf)))
        for name, f in variants:
            for _ in range(3):
                f()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(20):
                f()
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) / 20 * 1e3
            print(f"{name}: {us:.1f} us, {2.0 * a.m * D * D / us / 1e6:.1f} TFLOP/s")
    elif a.case == "verify_attention":
        B, Q, pool, hist = 4, 32, 4400, 3520
        kp = torch.randn(2 * pool, D, generator=g, device=dev).bfloat16()
        vp = torch.randn(2 * pool, D, generator=g, device=dev).bfloat16()
        qkv = torch.randn(B * Q, 3 * D, generator=g, device=dev).bfloat16()
        tl = [(s0, min(128, hist - s0)) for s0 in range(0, hist, 128)]
        tiles = torch.tensor(tl, dtype=torch.int32, device=dev).view(-1, 2)
        n = torch.tensor([len(tl)], dtype=torch.int32, device=dev)
        rows = torch.zeros(B, dtype=torch.int64, device=dev)
        out = torch.empty(B * Q, D, device=dev, dtype=torch.bfloat16)
        run = lambda: ops.attention(qkv, kp, vp, heads=H, q_rows=Q, src0_batch_stride=pool,  # noqa: E731
                                    tiles=tiles, n_tiles=n, src0_map=rows, k1=qkv, v1=qkv, k1_col=D,
                                    v1_col=2 * D, out=out)
    elif a.case == "attention":
        q = torch.randn(a.batch * a.q, D, generator=g, device=dev).bfloat16()
        kp = torch.randn(a.batch * a.pool, D, generator=g, device=dev).bfloat16()
        vp = torch.randn(a.batch * a.pool, D, generator=g, device=dev).bfloat16()
        out = torch.empty(a.batch * a.q, D, device=dev, dtype=torch.bfloat16)
        run = lambda: ops.attention(q, kp, vp, heads=H, q_rows=a.q, src0_batch_stride=a.pool,  # noqa: E731
                                    src0_len=a.pool, out=out)
    else:
        cfg = configs.PRESETS["cfg2"]
        blk = configs.build_blocks(configs.Config("p", D, H, F, 1, 1, (1, 16, 53), (8, 4, 1), 8), dev)[0]
        from wam_ops.native import NativeBlock
        nb = NativeBlock(blk)
        x = torch.randn(1, a.q, D, generator=g, device=dev).bfloat16()
        ctx = torch.randn(1, 8, D, generator=g, device=dev).bfloat16()
        temb = configs.make_temb(cfg, 1, dev, g)
        rope = configs.rope_freqs(torch.zeros(3, a.q)).to(dev)
        run = lambda: nb(x, ctx, temb, rope)  # noqa: E731
    for _ in range(3 + a.launches):
        run()
    torch.cuda.synchronize()
    code = _lib.device_status()
    print(f"{a.case}: ok, device status {code}")
    return 0 if code == 0 else 1


if __name__ == "__main__":
    sys.exit(main())
