"""Plain-PyTorch restatement of the reference Wan-DiT block (CPU, any dtype).

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py). Every class and function
cites the reference source it restates; paths are inside qingyiyi/WAM-egale:
  MODEL = 投机采样/wam-p0-worktree/wan_va/modules/model.py
  UTILS = 投机采样/wam-p0-worktree/wan_va/utils/utils.py
The module and parameter names match the reference so that the drop-in
installer (wam_ops.install.install_block) accepts these modules exactly as it
accepts the reference's own.
"""
import math

import torch
import torch.nn.functional as F
from torch import nn


def custom_sdpa(q, k, v):
    """MODEL:37-40. q,k,v [B, S, H, d] -> [B, Sq, H, d]; non-causal, scale 1/sqrt(d)."""
    out = F.scaled_dot_product_attention(q.transpose(1, 2), k.transpose(1, 2), v.transpose(1, 2))
    return out.transpose(1, 2)


class FP32LayerNorm(nn.LayerNorm):
    """diffusers FP32LayerNorm as used at MODEL:708,726-730,736: LayerNorm of
    the fp32-cast input with fp32 parameters, cast back to the input dtype
    (pinned by the reference's native restatement baseline/csrc/block.cu:279,289)."""

    def forward(self, inputs):
        origin = inputs.dtype
        return F.layer_norm(
            inputs.float(), self.normalized_shape,
            self.weight.float() if self.weight is not None else None,
            self.bias.float() if self.bias is not None else None, self.eps).to(origin)


class GELU(nn.Module):
    """diffusers GELU(dim, inner, approximate='tanh'): Linear then tanh-GELU
    (structure: 算子研究/…/block_baseline.py:105-109; formula block.cu:119-124)."""

    def __init__(self, dim_in, dim_out):
        super().__init__()
        self.proj = nn.Linear(dim_in, dim_out, bias=True)

    def forward(self, x):
        return F.gelu(self.proj(x), approximate="tanh")


class FeedForward(nn.Module):
    """diffusers FeedForward(dim, inner_dim=ffn_dim, activation_fn='gelu-approximate')
    (MODEL:733-735): net = [GELU(proj), Dropout(0), Linear(inner, dim)]."""

    def __init__(self, dim, inner_dim):
        super().__init__()
        self.net = nn.ModuleList([GELU(dim, inner_dim), nn.Dropout(0.0), nn.Linear(inner_dim, dim)])

    def forward(self, x):
        for m in self.net:
            x = m(x)
        return x


class WanRotaryPosEmbed(nn.Module):
    """MODEL:243-286: per-axis frequencies theta^(-2k/dim) for the f/h/w split
    (head_dim - 2*(head_dim//3), head_dim//3, head_dim//3) = 44/42/42 at 128;
    forward(grid_ids [B, 3+, L]) -> complex64 [B, L, head_dim/2]."""

    def __init__(self, attention_head_dim, theta=10000.0):
        super().__init__()
        self.attention_head_dim = attention_head_dim
        self.theta = theta
        self.f_dim = attention_head_dim - 2 * (attention_head_dim // 3)
        self.h_dim = attention_head_dim // 3
        self.w_dim = attention_head_dim // 3

        def base(d):
            return 1.0 / (theta ** (torch.arange(0, d, 2)[: d // 2].double() / d))

        self.f_freqs_base = base(self.f_dim)
        self.h_freqs_base = base(self.h_dim)
        self.w_freqs_base = base(self.w_dim)

    def forward(self, grid_ids):
        with torch.no_grad():
            f = grid_ids[:, 0, :].unsqueeze(-1) * self.f_freqs_base.to(grid_ids.device)
            h = grid_ids[:, 1, :].unsqueeze(-1) * self.h_freqs_base.to(grid_ids.device)
            w = grid_ids[:, 2, :].unsqueeze(-1) * self.w_freqs_base.to(grid_ids.device)
            freqs = torch.cat([f, h, w], dim=-1).float()
            return torch.polar(torch.ones_like(freqs), freqs)


def get_mesh_id(f, h, w, t, f_w=1, f_shift=0, action=False):
    """UTILS:33-54: (f, h, w, t) grid ids [4, f*h*w]; action tokens get
    fractional frame offsets and h = w = -1."""
    f_idx = torch.arange(f_shift, f + f_shift) * f_w
    ff, hh, ww = torch.meshgrid(f_idx, torch.arange(h), torch.arange(w), indexing="ij")
    if action:
        ff = ff + (torch.ones([h]).cumsum(0) / (h + 1)).view(1, -1, 1)
        hh = torch.ones_like(hh) * -1
        ww = torch.ones_like(ww) * -1
    grid = torch.cat([ff.unsqueeze(0), hh.unsqueeze(0), ww.unsqueeze(0)], dim=0).flatten(1)
    return torch.cat([grid, torch.full_like(grid[:1], t)], dim=0)


def apply_rotary_emb(x, freqs):
    """MODEL:616-621: rotate (even, odd) pairs by complex freqs in float64."""
    x_out = torch.view_as_complex(x.to(torch.float64).reshape(x.shape[0], x.shape[1], x.shape[2], -1, 2))
    x_out = torch.view_as_real(x_out * freqs).flatten(3)
    return x_out.to(x.dtype)


class WanAttention(nn.Module):
    """MODEL:289-691 with the "original" KV cache (the only mode the drop-in
    installer admits, install.py:22-23)."""

    def __init__(self, dim, heads, dim_head, eps=1e-6, cross_attention_dim_head=None,
                 attn_mode="torch"):
        super().__init__()
        if attn_mode != "torch":
            raise ValueError("the oracle restates the torch attention mode only")
        self.attn_op = custom_sdpa
        self.inner_dim = dim_head * heads
        self.heads = heads
        self.cross_attention_dim_head = cross_attention_dim_head
        self.kv_inner_dim = self.inner_dim if cross_attention_dim_head is None else cross_attention_dim_head * heads
        self.to_q = nn.Linear(dim, self.inner_dim, bias=True)
        self.to_k = nn.Linear(dim, self.kv_inner_dim, bias=True)
        self.to_v = nn.Linear(dim, self.kv_inner_dim, bias=True)
        self.to_out = nn.ModuleList([nn.Linear(self.inner_dim, dim, bias=True), nn.Dropout(0.0)])
        self.norm_q = nn.RMSNorm(dim_head * heads, eps=eps, elementwise_affine=True)
        self.norm_k = nn.RMSNorm(dim_head * heads, eps=eps, elementwise_affine=True)
        self.attn_caches = {} if cross_attention_dim_head is None else None
        self.cache_mode = "original"

    # ---------------------------------------------------------- KV cache
    def clear_pred_cache(self, cache_name):
        """MODEL:337-356 (original mode): drop prediction rows from the mask."""
        if self.attn_caches is None:
            return
        cache = self.attn_caches[cache_name]
        cache["mask"][cache["is_pred"]] = False

    def clear_cache(self, cache_name):
        if self.attn_caches is not None:
            self.attn_caches[cache_name] = None

    def init_kv_cache(self, cache_name, total_tolen, num_head, head_dim, device, dtype, batch_size):
        """MODEL:364-371 (original mode)."""
        if self.attn_caches is None:
            return
        self.attn_caches[cache_name] = self._original_cache(
            total_tolen, num_head, head_dim, device, dtype, batch_size)

    @staticmethod
    def _original_cache(total_tolen, num_head, head_dim, device, dtype, batch_size):
        """MODEL:417-434: K/V pool, int64 ids (-1 = never used), bool mask / is_pred."""
        return {
            "k": torch.empty([batch_size, total_tolen, num_head, head_dim], device=device, dtype=dtype),
            "v": torch.empty([batch_size, total_tolen, num_head, head_dim], device=device, dtype=dtype),
            "id": torch.full((total_tolen,), -1, device=device),
            "mask": torch.zeros((total_tolen,), dtype=torch.bool, device=device),
            "is_pred": torch.zeros((total_tolen,), dtype=torch.bool, device=device),
        }

    def allocate_slots(self, cache_name, key_size):
        """MODEL:547-566: the first `key_size` free slots in physical order;
        when too few are free, evict the used slots with the smallest ids
        first (stable: lower slot first among equal ids)."""
        cache = self.attn_caches[cache_name]
        mask, ids = cache["mask"], cache["id"]
        free = (~mask).nonzero(as_tuple=False).squeeze(-1)
        if free.numel() < key_size:
            used = mask.nonzero(as_tuple=False).squeeze(-1)
            order = torch.argsort(ids[used], stable=True)
            need = key_size - free.numel()
            to_free = used[order[:need]]
            mask[to_free] = False
            ids[to_free] = -1
            free = (~mask).nonzero(as_tuple=False).squeeze(-1)
        assert free.numel() >= key_size
        return free[:key_size]

    def _next_cache_id(self, cache_name):
        """MODEL:568-575."""
        ids = self.attn_caches[cache_name]["id"]
        mask = self.attn_caches[cache_name]["mask"]
        if mask.any():
            return ids[mask].max() + 1
        return torch.tensor(0, device=ids.device, dtype=ids.dtype)

    def update_cache(self, cache_name, key, value, is_pred):
        """MODEL:577-590."""
        cache = self.attn_caches[cache_name]
        slots = self.allocate_slots(cache_name, key.shape[1])
        new_id = self._next_cache_id(cache_name)
        cache["k"][:, slots] = key
        cache["v"][:, slots] = value
        cache["mask"][slots] = True
        cache["id"][slots] = new_id
        cache["is_pred"][slots] = is_pred
        return slots

    def restore_cache(self, cache_name, slots):
        """MODEL:592-593."""
        self.attn_caches[cache_name]["mask"][slots] = False

    # ----------------------------------------------------------- forward
    def forward(self, q, k, v, rotary_emb, update_cache=0, cache_name="pos", candidate_cache_rows=None):
        """MODEL:595-691 (original cache mode)."""
        kv_cache = (self.attn_caches[cache_name]
                    if self.attn_caches is not None and cache_name in self.attn_caches else None)
        query, key, value = self.to_q(q), self.to_k(k), self.to_v(v)
        query = self.norm_q(query).unflatten(2, (self.heads, -1))
        key = self.norm_k(key).unflatten(2, (self.heads, -1))
        value = value.unflatten(2, (self.heads, -1))
        if rotary_emb is not None:
            query = apply_rotary_emb(query, rotary_emb)
            key = apply_rotary_emb(key, rotary_emb)
        if candidate_cache_rows is not None:
            # MODEL:624-660: read-only history rows + each candidate's own K/V.
            if update_cache != 0 or kv_cache is None:
                raise ValueError("candidate verification requires existing read-only KV")
            valid = kv_cache["mask"].nonzero(as_tuple=False).squeeze(-1)
            history_key = kv_cache["k"][:, valid]
            history_value = kv_cache["v"][:, valid]
            rows = candidate_cache_rows
            if (rows.ndim != 1 or rows.numel() != query.shape[0] or rows.dtype != torch.long
                    or not bool(((rows >= 0) & (rows < history_key.shape[0])).all())):
                raise ValueError("invalid candidate_cache_rows for this KV cache")
            hidden = self.attn_op(query,
                                  torch.cat((history_key.index_select(0, rows), key), dim=1),
                                  torch.cat((history_value.index_select(0, rows), value), dim=1))
        else:
            # MODEL:667-686
            slots = None
            if kv_cache is not None and kv_cache["k"] is not None:
                slots = self.update_cache(cache_name, key, value, is_pred=(update_cache == 1))
                cache = self.attn_caches[cache_name]
                valid = cache["mask"].nonzero(as_tuple=False).squeeze(-1)
                key = cache["k"][:, valid]
                value = cache["v"][:, valid]
            hidden = self.attn_op(query, key, value)
            if update_cache == 0 and slots is not None:
                self.restore_cache(cache_name, slots)
        hidden = hidden.flatten(2, 3).type_as(query)
        hidden = self.to_out[0](hidden)
        return self.to_out[1](hidden)


class WanTransformerBlock(nn.Module):
    """MODEL:694-794."""

    def __init__(self, dim, ffn_dim, num_heads, cross_attn_norm=False, eps=1e-6, attn_mode="torch"):
        super().__init__()
        self.attn_mode = attn_mode
        self.norm1 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.attn1 = WanAttention(dim, num_heads, dim // num_heads, eps, None, attn_mode)
        self.attn2 = WanAttention(dim, num_heads, dim // num_heads, eps, dim // num_heads, attn_mode)
        self.norm2 = FP32LayerNorm(dim, eps, elementwise_affine=True) if cross_attn_norm else nn.Identity()
        self.ffn = FeedForward(dim, ffn_dim)
        self.norm3 = FP32LayerNorm(dim, eps, elementwise_affine=False)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 6, dim) / dim ** 0.5)

    def forward(self, hidden_states, encoder_hidden_states, temb, rotary_emb, update_cache=0,
                cache_name="pos", candidate_cache_rows=None):
        t = self.scale_shift_table[None] + temb.float()              # MODEL:751
        # 'b l n c -> b n l c' then chunk 6 along n (MODEL:752-759)
        shift_msa, scale_msa, gate_msa, c_shift, c_scale, c_gate = [
            t[:, :, i] for i in range(6)]
        norm = (self.norm1(hidden_states.float()) * (1.0 + scale_msa) + shift_msa).type_as(hidden_states)
        attn = self.attn1(norm, norm, norm, rotary_emb, update_cache=update_cache,
                          cache_name=cache_name, candidate_cache_rows=candidate_cache_rows)
        hidden_states = (hidden_states.float() + attn * gate_msa).type_as(hidden_states)   # MODEL:771-772
        norm = self.norm2(hidden_states.float()).type_as(hidden_states)                   # MODEL:775-776
        attn = self.attn2(norm, encoder_hidden_states, encoder_hidden_states, None,
                          update_cache=0, cache_name=cache_name)
        hidden_states = hidden_states + attn                                               # MODEL:783
        norm = (self.norm3(hidden_states.float()) * (1.0 + c_scale) + c_shift).type_as(hidden_states)
        ff = self.ffn(norm)                                                                # MODEL:790
        return (hidden_states.float() + ff.float() * c_gate).type_as(hidden_states)        # MODEL:792-793


def stack_forward(blocks, hidden_states, context, temb, rotary_emb, update_cache=0,
                  cache_name="pos", candidate_cache_rows=None):
    """The 30-block loop of WanTransformer3DModel.forward (MODEL:1091-1098)."""
    for block in blocks:
        hidden_states = block(hidden_states, context, temb, rotary_emb, update_cache=update_cache,
                              cache_name=cache_name, candidate_cache_rows=candidate_cache_rows)
    return hidden_states
