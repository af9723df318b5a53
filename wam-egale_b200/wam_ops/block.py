"""Parameter/cache containers whose forward is the B200 native block.

Mirrors 算子研究/wam_ops/baseline/block.py:10-78 and baseline/attention.py:6-45:
the classes keep the reference module structure and state_dict names
(norm1, attn1.{to_q,to_k,to_v,to_out.0,norm_q,norm_k}, attn2.*, norm2, ffn.net.{0.proj,2},
norm3, scale_shift_table) and the "original" KV-cache API, while
`TransformerBlock.forward` runs the whole block in libwamb.so.
`install_block` swaps a reference block's classes to these in place.
"""
import torch
from torch import nn
import torch.nn.functional as F

from .native import NativeBlock


class FP32LayerNorm(nn.LayerNorm):
    """Parameter container matching diffusers FP32LayerNorm (weights only)."""


class _GELUProj(nn.Module):
    def __init__(self, dim_in, dim_out):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out, bias=True)


class FeedForward(nn.Module):
    """Parameter container with the diffusers FeedForward layout: net.0.proj, net.2."""

    def __init__(self, dim, inner_dim):
        super().__init__()
        self.net = nn.ModuleList([_GELUProj(dim, inner_dim), nn.Dropout(0.0), nn.Linear(inner_dim, dim)])


class Attention(nn.Module):
    """WanAttention parameters + the "original" KV cache (model.py:289-593).
    Forward is not available on its own: the block forward is native."""

    def __init__(self, dim, heads=8, dim_head=64, eps=1e-5, dropout=0.0,
                 cross_attention_dim_head=None, attn_mode="torch"):
        super().__init__()
        if attn_mode != "torch":
            raise ValueError("the native block accepts the torch attention parameter protocol only")
        self.attn_mode = attn_mode
        self.inner_dim = dim_head * heads
        self.heads = heads
        self.cross_attention_dim_head = cross_attention_dim_head
        self.kv_inner_dim = self.inner_dim if cross_attention_dim_head is None else cross_attention_dim_head * heads
        self.to_q = nn.Linear(dim, self.inner_dim, bias=True)
        self.to_k = nn.Linear(dim, self.kv_inner_dim, bias=True)
        self.to_v = nn.Linear(dim, self.kv_inner_dim, bias=True)
        self.to_out = nn.ModuleList([nn.Linear(self.inner_dim, dim, bias=True), nn.Dropout(dropout)])
        self.norm_q = nn.RMSNorm(dim_head * heads, eps=eps, elementwise_affine=True)
        self.norm_k = nn.RMSNorm(dim_head * heads, eps=eps, elementwise_affine=True)
        self.attn_caches = {} if cross_attention_dim_head is None else None
        self.cache_mode = "original"

    def clear_pred_cache(self, cache_name):
        if self.attn_caches is not None:
            cache = self.attn_caches[cache_name]
            cache["mask"][cache["is_pred"]] = False

    def clear_cache(self, cache_name):
        if self.attn_caches is not None:
            self.attn_caches[cache_name] = None

    def init_kv_cache(self, cache_name, total_tolen, num_head, head_dim, device, dtype, batch_size):
        if self.attn_caches is not None:
            self.attn_caches[cache_name] = self._original_cache(
                total_tolen, num_head, head_dim, device, dtype, batch_size)

    @staticmethod
    def _original_cache(total_tolen, num_head, head_dim, device, dtype, batch_size):
        return {
            "k": torch.empty([batch_size, total_tolen, num_head, head_dim], device=device, dtype=dtype),
            "v": torch.empty([batch_size, total_tolen, num_head, head_dim], device=device, dtype=dtype),
            "id": torch.full((total_tolen,), -1, device=device),
            "mask": torch.zeros((total_tolen,), dtype=torch.bool, device=device),
            "is_pred": torch.zeros((total_tolen,), dtype=torch.bool, device=device),
        }

    def forward(self, *args, **kwargs):
        raise RuntimeError("Attention is a parameter/cache container; call the native TransformerBlock")


class TransformerBlock(nn.Module):
    """WanTransformerBlock parameters (model.py:694-739); forward runs natively."""
    attention_cls = Attention
    native_fused_ffn1 = False
    execution_mode = "sequential"

    def __init__(self, dim, ffn_dim, num_heads, cross_attn_norm=False, eps=1e-6, attn_mode="torch"):
        super().__init__()
        self.attn_mode = attn_mode
        self.norm1 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.attn1 = self.attention_cls(dim=dim, heads=num_heads, dim_head=dim // num_heads, eps=eps,
                                        cross_attention_dim_head=None, attn_mode=attn_mode)
        self.attn2 = self.attention_cls(dim=dim, heads=num_heads, dim_head=dim // num_heads, eps=eps,
                                        cross_attention_dim_head=dim // num_heads, attn_mode=attn_mode)
        self.norm2 = FP32LayerNorm(dim, eps, elementwise_affine=True) if cross_attn_norm else nn.Identity()
        self.ffn = FeedForward(dim, ffn_dim)
        self.norm3 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)

    def forward(self, hidden_states, encoder_hidden_states, temb, rotary_emb, update_cache=0,
                cache_name="pos", candidate_cache_rows=None):
        native = self.__dict__.get("_native_block")
        if native is None:
            native = NativeBlock(self, fused_ffn1=self.native_fused_ffn1, mode=self.execution_mode)
            object.__setattr__(self, "_native_block", native)
        return native(hidden_states, encoder_hidden_states, temb, rotary_emb,
                      update_cache, cache_name, candidate_cache_rows)
