"""CPU checks of the FP8 model in oracle/fp8.py (the GPU comparison is in
test_gpu_fp8.py): E4M3 rounding is round-to-nearest-even with saturation at
448, the row scale maps each row's largest magnitude to 448, the per-row
reciprocal is a correctly rounded division, and an fp8 block stays close to
the unquantized one."""
import torch

from blockutil import make_inputs, make_oracle_block, stats
from oracle import fp8 as of8


def test_e4m3_round_to_nearest_even():
    v = torch.tensor([1.0625, 1.1875, 90.6, 84.0, 84.00001, 2.0 ** -10, 1.5 * 2.0 ** -9, 448.0])
    want = torch.tensor([1.0, 1.25, 88.0, 80.0, 88.0, 0.0, 2.0 ** -8, 448.0])
    assert torch.equal(v.to(torch.float8_e4m3fn).float(), want)


def test_quant_rows_scale_and_reciprocal():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(300, 512, generator=g) * torch.logspace(-3, 3, 300)[:, None]
    x[7] = 0
    q, s = of8.quant_rows(x)
    amax = x.abs().amax(-1).clamp_min(1e-20)
    exact_inv = torch.tensor([448.0 / v for v in amax.double().tolist()], dtype=torch.float64).float()
    assert torch.equal((x * exact_inv[:, None]).to(torch.float8_e4m3fn).view(torch.uint8), q.view(torch.uint8))
    assert torch.equal(s, amax / 448.0)
    assert torch.equal(q.float().abs().amax(-1)[torch.arange(300) != 7], torch.full((299,), 448.0))
    err = (of8.dequant(q, s) - x).abs() / amax[:, None]
    assert err.max() <= 16.0 / 448.0  # half an E4M3 step of the top binade [256, 448], over amax


def test_fp8_block_close_to_exact():
    blk = make_oracle_block(256, 512, 2, seed=1)
    x, ctx, temb, rope = make_inputs(1, 48, 256, 32, 2, seed=3)
    with torch.no_grad():
        s = stats(of8.fp8_block(blk)(x, ctx, temb, rope), blk(x, ctx, temb, rope))
    assert s["cos"] > 0.9999 and s["max_abs"] < 0.1, s
