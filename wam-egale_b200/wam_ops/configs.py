"""Named presets of the benchmark configurations and their seeded synthetic
inputs (the reference has no public dataset on this path; weights and inputs
are synthetic with the shapes and distributions the configs state).

  cfg0  one block, D 1536 / 12x128 heads / FFN 8960, 1560 video (2x30x26) +
        32 action tokens, 512 context tokens (fp32 CPU oracle case)
  cfg1  30 x cfg0 blocks, bf16, cross K/V prepared
  cfg2  30 layers, D 3072 / 24x128 / FFN 14336; KV pool of 5 x 880 slots
        holding 4 history chunks (3520 tokens), one 880-token chunk (848 video
        + 32 action) denoised with update_cache=0; 512 context tokens
  cfg3  cfg2 stack, 4 candidate chunks x 32 tokens verified against the
        read-only 3520-token history (candidate_cache_rows = [0, 0, 0, 0])
  cfg4  cfg2 x 64 rollouts, 8 per GPU (batch 8 per rank)

Weights: Linear N(0, 0.02), biases 0, RMSNorm / LayerNorm gains 1 and
shifts 0, scale_shift_table randn / sqrt(D) (model.py:738-739). temb comes
from t ~ U[0, 1000) through the 256-d sinusoidal embedding (flip_sin_to_cos,
shift 0) and Linear-SiLU-Linear, SiLU, Linear(D, 6D) (model.py:203-240); this
timestep chain is outside the block and its diffusers source is not in the
reference tree, so it only has to be a plausible temb generator.
"""
import math
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class Config:
    name: str
    dim: int
    heads: int
    ffn: int
    layers: int
    batch: int
    video: tuple          # (f, h, w) grid of the chunk's video tokens
    action: tuple         # (f, h, w) grid of the action tokens (get_mesh_id action=True)
    context: int
    history_chunks: int = 0
    pool_chunks: int = 0
    candidates: int = 0

    @property
    def tokens(self):
        return math.prod(self.video) + math.prod(self.action)


PRESETS = {
    "cfg0": Config("cfg0", 1536, 12, 8960, 1, 1, (2, 30, 26), (8, 4, 1), 512),
    "cfg1": Config("cfg1", 1536, 12, 8960, 30, 1, (2, 30, 26), (8, 4, 1), 512),
    "cfg2": Config("cfg2", 3072, 24, 14336, 30, 1, (1, 16, 53), (8, 4, 1), 512, 4, 5),
    "cfg3": Config("cfg3", 3072, 24, 14336, 30, 4, (0, 0, 0), (8, 4, 1), 512, 4, 5, candidates=4),
    "cfg4": Config("cfg4", 3072, 24, 14336, 30, 8, (1, 16, 53), (8, 4, 1), 512, 4, 5),
}


def mesh_id(f, h, w, t, f_shift=0, action=False):
    """get_mesh_id (投机采样/wam-p0-worktree/wan_va/utils/utils.py:33-54)."""
    ff, hh, ww = torch.meshgrid(torch.arange(f_shift, f + f_shift).float(), torch.arange(h).float(),
                                torch.arange(w).float(), indexing="ij")
    if action:
        ff = ff + (torch.ones([h]).cumsum(0) / (h + 1)).view(1, -1, 1)
        hh = torch.full_like(hh, -1.0)
        ww = torch.full_like(ww, -1.0)
    grid = torch.stack([ff, hh, ww]).flatten(1)
    return torch.cat([grid, torch.full_like(grid[:1], t)], 0)


def rope_freqs(grid, head_dim=128, theta=10000.0):
    """WanRotaryPosEmbed.forward (model.py:243-286): complex64 [1, L, 1, 64]."""
    f_dim = head_dim - 2 * (head_dim // 3)
    hw = head_dim // 3

    def base(d):
        return 1.0 / (theta ** (torch.arange(0, d, 2, device=grid.device)[: d // 2].double() / d))

    parts = [grid[0][:, None].double() * base(f_dim), grid[1][:, None].double() * base(hw),
             grid[2][:, None].double() * base(hw)]
    freqs = torch.cat(parts, -1).float()
    return torch.polar(torch.ones_like(freqs), freqs)[None, :, None]


def chunk_rope(cfg, f_shift=0):
    grids = []
    if math.prod(cfg.video):
        grids.append(mesh_id(*cfg.video, 0, f_shift=f_shift))
    grids.append(mesh_id(*cfg.action, 0, f_shift=f_shift, action=True))
    return rope_freqs(torch.cat(grids, 1))


def timestep_embedding(t, dim=256):
    """Sinusoidal embedding, cos first (flip_sin_to_cos=True, shift 0)."""
    half = dim // 2
    freqs = torch.exp(-math.log(10000.0) * torch.arange(half, dtype=torch.float32, device=t.device) / half)
    arg = t.float()[:, None] * freqs[None]
    return torch.cat([torch.cos(arg), torch.sin(arg)], -1)


def make_temb(cfg, batch, device, gen, per_token=1):
    """temb [batch, per_token, 6, D] fp32 from t ~ U[0, 1000) (seeded)."""
    D = cfg.dim
    t = torch.rand(batch * per_token, generator=gen, device=device) * 1000.0
    w1 = torch.randn(D, 256, generator=gen, device=device) * 0.02
    w2 = torch.randn(D, D, generator=gen, device=device) * 0.02
    w3 = torch.randn(6 * D, D, generator=gen, device=device) * 0.02
    e = timestep_embedding(t) @ w1.t()
    e = torch.nn.functional.silu(e) @ w2.t()
    proj = torch.nn.functional.silu(e) @ w3.t()
    return proj.view(batch, per_token, 6, D).contiguous()


def build_blocks(cfg, device, seed=0):
    """cfg.layers native-block containers with seeded weights on `device`."""
    from .block import TransformerBlock

    gen = torch.Generator(device=device).manual_seed(seed)
    blocks = []
    for _ in range(cfg.layers):
        with torch.device("meta"):
            blk = TransformerBlock(cfg.dim, cfg.ffn, cfg.heads, cross_attn_norm=True, eps=1e-6)
        blk = blk.to_empty(device=device)
        with torch.no_grad():
            for name, p in blk.named_parameters():
                if name.endswith("scale_shift_table"):
                    p.data = (torch.randn(p.shape, generator=gen, device=device) / cfg.dim ** 0.5).float()
                elif name.startswith("norm2"):
                    p.data = (torch.ones(p.shape, device=device) if name.endswith("weight")
                              else torch.zeros(p.shape, device=device)).float()
                elif "norm_q" in name or "norm_k" in name:
                    p.data = torch.ones(p.shape, device=device, dtype=torch.bfloat16)
                elif name.endswith("weight"):
                    p.data = (torch.randn(p.shape, generator=gen, device=device,
                                          dtype=torch.bfloat16) * 0.02).contiguous()
                else:
                    p.data = torch.zeros(p.shape, device=device, dtype=torch.bfloat16)
        blocks.append(blk.eval())
    return blocks


def fill_history(blocks, cfg, device, gen, pool_batch):
    """Pre-filled self-KV pool: history_chunks x tokens slots with ids
    0..history_chunks-1, random K/V of unit scale (the magnitude of
    RMS-normalised keys), pool = pool_chunks x tokens slots."""
    Q = cfg.tokens if not cfg.candidates else PRESETS["cfg2"].tokens
    pool = cfg.pool_chunks * Q
    hist = cfg.history_chunks * Q
    for blk in blocks:
        blk.attn1.init_kv_cache("pos", pool, cfg.heads, 128, device, torch.bfloat16, pool_batch)
        c = blk.attn1.attn_caches["pos"]
        c["k"].normal_(generator=gen)
        c["v"].normal_(generator=gen)
        c["mask"][:hist] = True
        c["id"][:hist] = torch.arange(hist, device=device) // Q
    return pool, hist


def build_model(cfg, device, seed=0, text_dim=4096, action_dim=30, in_channels=48):
    """A WanModel container (embedders, cfg.layers blocks, output head) with
    seeded weights on `device`: Linear weights N(0, 0.02) bf16, biases 0,
    tables randn / sqrt(D) fp32, norm gains 1 (the timestep embedder fp32, as
    the reference keeps it, model.py:812-825)."""
    from .model import WanModel

    gen = torch.Generator(device=device).manual_seed(seed)
    with torch.device("meta"):
        m = WanModel(num_attention_heads=cfg.heads, in_channels=in_channels, out_channels=in_channels,
                     action_dim=action_dim, text_dim=text_dim, ffn_dim=cfg.ffn, num_layers=cfg.layers)
    m = m.to_empty(device=device)
    with torch.no_grad():
        for name, p in m.named_parameters():
            fp32 = name.endswith("scale_shift_table") or "norm2" in name or "time_embedder" in name
            if name.endswith("scale_shift_table"):
                v = torch.randn(p.shape, generator=gen, device=device) / cfg.dim ** 0.5
            elif "norm" in name and name.endswith("weight"):
                v = torch.ones(p.shape, device=device)
            elif name.endswith("weight"):
                v = torch.randn(p.shape, generator=gen, device=device) * 0.02
            else:
                v = torch.zeros(p.shape, device=device)
            p.data = v.to(torch.float32 if fp32 else torch.bfloat16).contiguous()
    return m.eval()
