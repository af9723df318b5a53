"""Plain-PyTorch restatement of the whole-model inference forward around the
block stack, and of the flow-match scheduler -- TEST INFRASTRUCTURE ONLY (see
oracle/__init__.py). Paths are inside qingyiyi/WAM-egale:
  MODEL = 投机采样/wam-p0-worktree/wan_va/modules/model.py
  SCHED = 投机采样/wam-p0-worktree/wan_va/utils/scheduler.py

The diffusers modules the model imports (Timesteps, TimestepEmbedding,
PixArtAlphaTextProjection; diffusers is not in the reference tree nor
installed) are restated from their published definitions; module and
parameter names follow the reference so that state_dicts load unchanged.
"""
import math
from copy import deepcopy

import torch
import torch.nn.functional as F
from einops import rearrange
from torch import nn

from . import wan_block as ob


class Timesteps(nn.Module):
    """diffusers Timesteps / get_timestep_embedding (scale 1, max_period
    10000): exponent_i = -ln(10000) i / (half - shift); [sin, cos], swapped to
    [cos, sin] by flip_sin_to_cos (used at MODEL:213-215)."""

    def __init__(self, num_channels, flip_sin_to_cos=True, downscale_freq_shift=0):
        super().__init__()
        self.num_channels, self.flip, self.shift = num_channels, flip_sin_to_cos, downscale_freq_shift

    def forward(self, t):
        half = self.num_channels // 2
        exponent = -math.log(10000) * torch.arange(half, dtype=torch.float32, device=t.device)
        exponent = exponent / (half - self.shift)
        emb = t[:, None].float() * torch.exp(exponent)[None, :]
        emb = torch.cat([torch.sin(emb), torch.cos(emb)], dim=-1)
        if self.flip:
            emb = torch.cat([emb[:, half:], emb[:, :half]], dim=-1)
        return emb


class TimestepEmbedding(nn.Module):
    """diffusers TimestepEmbedding: linear_1, SiLU, linear_2 (MODEL:216-217)."""

    def __init__(self, in_channels, time_embed_dim):
        super().__init__()
        self.linear_1 = nn.Linear(in_channels, time_embed_dim)
        self.act = nn.SiLU()
        self.linear_2 = nn.Linear(time_embed_dim, time_embed_dim)

    def forward(self, x):
        return self.linear_2(self.act(self.linear_1(x)))


class PixArtAlphaTextProjection(nn.Module):
    """diffusers PixArtAlphaTextProjection(act_fn="gelu_tanh"): linear_1,
    tanh-GELU, linear_2 (MODEL:220-222)."""

    def __init__(self, in_features, hidden_size):
        super().__init__()
        self.linear_1 = nn.Linear(in_features, hidden_size)
        self.act_1 = nn.GELU(approximate="tanh")
        self.linear_2 = nn.Linear(hidden_size, hidden_size)

    def forward(self, x):
        return self.linear_2(self.act_1(self.linear_1(x)))


class WanTimeTextImageEmbedding(nn.Module):
    """MODEL:203-240."""

    def __init__(self, dim, time_freq_dim, time_proj_dim, text_embed_dim):
        super().__init__()
        self.timesteps_proj = Timesteps(time_freq_dim, True, 0)
        self.time_embedder = TimestepEmbedding(time_freq_dim, dim)
        self.act_fn = nn.SiLU()
        self.time_proj = nn.Linear(dim, time_proj_dim)
        self.text_embedder = PixArtAlphaTextProjection(text_embed_dim, dim)

    def forward(self, timestep, dtype=None):
        B, L = timestep.shape
        timestep = self.timesteps_proj(timestep.reshape(-1))
        wdt = self.time_embedder.linear_1.weight.dtype
        if timestep.dtype != wdt:
            timestep = timestep.to(wdt)
        temb = self.time_embedder(timestep).to(dtype=dtype)
        timestep_proj = self.time_proj(self.act_fn(temb))
        return temb.reshape(B, L, -1), timestep_proj.reshape(B, L, -1)


class WanTransformer3DModel(nn.Module):
    """MODEL:797-872 (construction) and the inference branch of
    MODEL:1028-1116 (forward with train_mode=False)."""

    def __init__(self, patch_size=(1, 2, 2), num_attention_heads=24, attention_head_dim=128,
                 in_channels=48, out_channels=48, action_dim=30, text_dim=4096, freq_dim=256,
                 ffn_dim=14336, num_layers=30, cross_attn_norm=True, eps=1e-6):
        super().__init__()
        self.patch_size = list(patch_size)
        inner = num_attention_heads * attention_head_dim
        self.num_attention_heads, self.attention_head_dim = num_attention_heads, attention_head_dim
        self.rope = ob.WanRotaryPosEmbed(attention_head_dim)
        self.patch_embedding_mlp = nn.Linear(in_channels * math.prod(patch_size), inner)
        self.action_embedder = nn.Linear(action_dim, inner)
        self.condition_embedder = WanTimeTextImageEmbedding(inner, freq_dim, inner * 6, text_dim)
        self.condition_embedder_action = deepcopy(self.condition_embedder)
        self.blocks = nn.ModuleList([ob.WanTransformerBlock(inner, ffn_dim, num_attention_heads,
                                                            cross_attn_norm, eps)
                                     for _ in range(num_layers)])
        self.norm_out = ob.FP32LayerNorm(inner, eps, elementwise_affine=False)
        self.proj_out = nn.Linear(inner, out_channels * math.prod(patch_size))
        self.action_proj_out = nn.Linear(inner, action_dim)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 2, inner) / inner ** 0.5)

    def forward(self, input_dict, update_cache=0, cache_name="pos", action_mode=False,
                candidate_cache_rows=None):
        if candidate_cache_rows is not None and update_cache != 0:
            raise ValueError("candidate read-only forward requires inference and update_cache=0")
        x = input_dict["noisy_latents"]
        if action_mode:                                                   # MODEL:1063-1066
            h = self.action_embedder(rearrange(x, "b c f h w -> b (f h w) c"))
        else:                                                             # MODEL:1067-1077
            p1, p2, p3 = self.patch_size
            h = self.patch_embedding_mlp(rearrange(
                x, "b c (f p1) (h p2) (w p3) -> b (f h w) (c p1 p2 p3)", p1=p1, p2=p2, p3=p3))
        text = self.condition_embedder.text_embedder(input_dict["text_emb"])   # MODEL:1078-1079
        rotary_emb = self.rope(input_dict["grid_id"])[:, :, None]              # MODEL:1081-1082
        ph, pw = (1, 1) if action_mode else (self.patch_size[1], self.patch_size[2])
        steps = torch.repeat_interleave(input_dict["timesteps"],
                                        (x.shape[-2] // ph) * (x.shape[-1] // pw), dim=1)  # MODEL:1086-1089
        emb = self.condition_embedder_action if action_mode else self.condition_embedder
        temb, timestep_proj = emb(steps, dtype=h.dtype)
        timestep_proj = timestep_proj.unflatten(2, (6, -1))
        for block in self.blocks:                                         # MODEL:1095-1102
            h = block(h, text, timestep_proj, rotary_emb, update_cache=update_cache,
                      cache_name=cache_name, candidate_cache_rows=candidate_cache_rows)
        tab = self.scale_shift_table[None] + temb[:, :, None, ...]         # MODEL:1103-1110
        shift, scale = rearrange(tab, "b l n c -> b n l c").chunk(2, dim=1)
        shift, scale = shift.squeeze(1), scale.squeeze(1)
        h = (self.norm_out(h.float()) * (1.0 + scale) + shift).type_as(h)
        if action_mode:                                                   # MODEL:1112-1118
            return self.action_proj_out(h)
        h = self.proj_out(h)
        return rearrange(h, "b l (n c) -> b (l n) c", n=math.prod(self.patch_size))


class FlowMatchScheduler:
    """SCHED:6-89 (inference: set_timesteps without training weights, step)."""

    def __init__(self, num_inference_steps=100, num_train_timesteps=1000, shift=3.0, sigma_max=1.0,
                 sigma_min=0.003 / 1.002, inverse_timesteps=False, extra_one_step=False,
                 reverse_sigmas=False):
        self.num_train_timesteps, self.shift = num_train_timesteps, shift
        self.sigma_max, self.sigma_min = sigma_max, sigma_min
        self.inverse_timesteps, self.extra_one_step = inverse_timesteps, extra_one_step
        self.reverse_sigmas = reverse_sigmas
        self.set_timesteps(num_inference_steps)

    def set_timesteps(self, num_inference_steps=100, denoising_strength=1.0, shift=None):
        if shift is not None:
            self.shift = shift
        start = self.sigma_min + (self.sigma_max - self.sigma_min) * denoising_strength
        if self.extra_one_step:
            self.sigmas = torch.linspace(start, self.sigma_min, num_inference_steps + 1)[:-1]
        else:
            self.sigmas = torch.linspace(start, self.sigma_min, num_inference_steps)
        if self.inverse_timesteps:
            self.sigmas = torch.flip(self.sigmas, dims=[0])
        self.sigmas = self.shift * self.sigmas / (1 + (self.shift - 1) * self.sigmas)
        if self.reverse_sigmas:
            self.sigmas = 1 - self.sigmas
        self.timesteps = self.sigmas * self.num_train_timesteps

    def step(self, model_output, timestep, sample, to_final=False):
        timestep_id = torch.argmin((self.timesteps - float(timestep)).abs())
        sigma = self.sigmas[timestep_id]
        if to_final or timestep_id + 1 >= len(self.timesteps):
            sigma_ = 1 if (self.inverse_timesteps or self.reverse_sigmas) else 0
        else:
            sigma_ = self.sigmas[timestep_id + 1]
        return sample + model_output * (sigma_ - sigma)
