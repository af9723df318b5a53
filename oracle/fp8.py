"""CPU model of the FP8-E4M3 path -- TEST INFRASTRUCTURE ONLY (see
oracle/__init__.py).

The reference has no FP8 path (it is bf16-only: 算子研究/wam_ops/baseline/
csrc/gemm.h:36-38), so there is nothing to pin this against; it restates the
quantization scheme the B200 build implements, on top of the fp32 block
restatement in wan_block.py:

* row quantization (activations per token, weights per output channel):
    amax = max(max |x[r]|, 1e-20); q = e4m3_rne(x * (448 / amax)); scale = amax / 448
* the eight step GEMMs (self q/k/v/out, cross q/out, FFN proj/out) compute
    y = (q_a * s_a) @ (q_w * s_w)^T + b        in fp32
* GEMM inputs that the GPU stores as bf16 before quantizing (attention
  outputs, GELU output) are rounded to bf16 first; LayerNorm outputs are
  quantized straight from fp32. Cross K/V projections stay unquantized.
"""
import copy

import torch
from torch import nn


def quant_rows(x):
    """Row-wise E4M3 quantization of a 2-D tensor: (q float8_e4m3fn, scale fp32 [rows])."""
    x = x.float()
    amax = x.abs().amax(dim=-1).clamp_min(1e-20)
    c448 = torch.full_like(amax, 448.0)
    # tensor / tensor: a correctly rounded fp32 division like the GPU's
    # (torch evaluates `scalar / tensor` as scalar * reciprocal(tensor), which
    # can differ in the last bit).
    q = (x * (c448 / amax)[:, None]).to(torch.float8_e4m3fn)
    return q, amax / c448


def dequant(q, scale):
    return q.float() * scale[:, None]


class QuantLinear(nn.Module):
    """nn.Linear with an E4M3 per-channel weight and per-token E4M3 input."""

    def __init__(self, lin, round_input_bf16):
        super().__init__()
        q, s = quant_rows(lin.weight.detach())
        self.register_buffer("w", dequant(q, s))
        self.register_buffer("b", lin.bias.detach().float())
        self.round_input_bf16 = round_input_bf16

    def forward(self, x):
        shape = x.shape
        x = x.float().reshape(-1, shape[-1])
        if self.round_input_bf16:
            x = x.bfloat16().float()
        q, s = quant_rows(x)
        y = dequant(q, s) @ self.w.t() + self.b
        return y.reshape(*shape[:-1], -1)


def fp8_block(block):
    """A copy of an oracle WanTransformerBlock whose eight step GEMMs follow
    the FP8 path (the copy shares nothing with `block` but the KV cache
    tensors it deep-copies)."""
    b = copy.deepcopy(block)
    for name in ("to_q", "to_k", "to_v"):
        setattr(b.attn1, name, QuantLinear(getattr(block.attn1, name), False))
    b.attn1.to_out[0] = QuantLinear(block.attn1.to_out[0], True)
    b.attn2.to_q = QuantLinear(block.attn2.to_q, False)
    b.attn2.to_out[0] = QuantLinear(block.attn2.to_out[0], True)
    b.ffn.net[0].proj = QuantLinear(block.ffn.net[0].proj, False)
    b.ffn.net[2] = QuantLinear(block.ffn.net[2], True)
    return b
