"""The whole-model inference forward around the native block stack.

NativeWanModel runs WanTransformer3DModel.forward (投机采样/wam-p0-worktree/
wan_va/modules/model.py:1028-1116, inference branch) on the device: the
latent patchify / action input embedding, the text projection, the timestep
embedding chain (diffusers Timesteps + TimestepEmbedding, time_proj), the 30
blocks (NativeStack, fp32 residual stream between them), the output norm
with its modulation and the output projection -- every GEMM on the tcgen05
kernel and the glue in libwamb.so (wamb_embed_gather, wamb_timestep_embedding,
wamb_silu, wamb_repeat_rows, wamb_output_norm, wamb_copy_cols). It binds a
model whose modules carry the reference's names (the reference's own model,
or WanModel below).

Numerics: the reference keeps the timestep embedder in fp32; here its GEMMs
take bf16 operands with fp32 accumulation, and its output (temb) stays fp32.
The timestep embedding is computed once per distinct timestep row and then
repeated to every token (the reference embeds the repeated rows).
"""
import math
from copy import deepcopy

import torch
from torch import nn

from . import _lib, ops
from .block import FP32LayerNorm, TransformerBlock
from .configs import rope_freqs
from .stack import NativeStack


def _ceil64(n):
    return (n + 63) // 64 * 64


def _bf16(t):
    return t.detach().to(torch.bfloat16).contiguous()


def _pad_cols(w, k):
    """[N, K0] -> [N, k] bf16, zero columns after K0."""
    out = torch.zeros(w.shape[0], k, dtype=torch.bfloat16, device=w.device)
    out[:, : w.shape[1]] = w.detach()
    return out


def _pad_rows(w, b, n):
    """[N0, K] weight and [N0] bias -> n rows (zero rows after N0)."""
    wo = torch.zeros(n, w.shape[1], dtype=torch.bfloat16, device=w.device)
    bo = torch.zeros(n, dtype=torch.bfloat16, device=w.device)
    wo[: w.shape[0]] = w.detach()
    bo[: b.shape[0]] = b.detach()
    return wo, bo


class _TimeEmbedding(nn.Module):
    def __init__(self, freq_dim, dim, text_dim):
        super().__init__()
        self.time_embedder = nn.Module()
        self.time_embedder.linear_1 = nn.Linear(freq_dim, dim)
        self.time_embedder.linear_2 = nn.Linear(dim, dim)
        self.time_proj = nn.Linear(dim, dim * 6)
        self.text_embedder = nn.Module()
        self.text_embedder.linear_1 = nn.Linear(text_dim, dim)
        self.text_embedder.linear_2 = nn.Linear(dim, dim)


class WanModel(nn.Module):
    """Parameter container with the WanTransformer3DModel layout and names
    (model.py:797-872): patch_embedding_mlp, action_embedder,
    condition_embedder{,_action}.{time_embedder.linear_1/2, time_proj,
    text_embedder.linear_1/2}, blocks, norm_out, proj_out, action_proj_out,
    scale_shift_table. Its forward is NativeWanModel."""

    def __init__(self, patch_size=(1, 2, 2), num_attention_heads=24, attention_head_dim=128,
                 in_channels=48, out_channels=48, action_dim=30, text_dim=4096, freq_dim=256,
                 ffn_dim=14336, num_layers=30, cross_attn_norm=True, eps=1e-6):
        super().__init__()
        inner = num_attention_heads * attention_head_dim
        self.patch_size = list(patch_size)
        self.num_attention_heads, self.attention_head_dim = num_attention_heads, attention_head_dim
        self.patch_embedding_mlp = nn.Linear(in_channels * math.prod(patch_size), inner)
        self.action_embedder = nn.Linear(action_dim, inner)
        self.condition_embedder = _TimeEmbedding(freq_dim, inner, text_dim)
        self.condition_embedder_action = deepcopy(self.condition_embedder)
        self.blocks = nn.ModuleList([TransformerBlock(inner, ffn_dim, num_attention_heads,
                                                      cross_attn_norm=cross_attn_norm, eps=eps)
                                     for _ in range(num_layers)])
        self.norm_out = FP32LayerNorm(inner, eps, elementwise_affine=False)
        self.proj_out = nn.Linear(inner, out_channels * math.prod(patch_size))
        self.action_proj_out = nn.Linear(inner, action_dim)
        self.scale_shift_table = nn.Parameter(torch.randn(1, 2, inner) / inner ** 0.5)


class _Embedders:
    """bf16 GEMM operands of one WanTimeTextImageEmbedding."""

    def __init__(self, m):
        te, tx = m.time_embedder, m.text_embedder
        self.t1 = (_bf16(te.linear_1.weight), _bf16(te.linear_1.bias))
        self.t2 = (_bf16(te.linear_2.weight), _bf16(te.linear_2.bias))
        self.tp = (_bf16(m.time_proj.weight), _bf16(m.time_proj.bias))
        self.x1 = (_bf16(tx.linear_1.weight), _bf16(tx.linear_1.bias))
        self.x2 = (_bf16(tx.linear_2.weight), _bf16(tx.linear_2.bias))
        self.freq_dim = te.linear_1.weight.shape[1]


class NativeWanModel:
    def __init__(self, model, fp8=False):
        self.model = model
        D = model.scale_shift_table.shape[-1]
        self.dim = D
        self.patch_size = list(model.patch_size)
        self.stack = NativeStack(list(model.blocks), fp8=fp8)
        self.eps = float(getattr(model.norm_out, "eps", 1e-6))
        self.table = model.scale_shift_table.detach().float().reshape(2, D).contiguous()
        pe, ae = model.patch_embedding_mlp, model.action_embedder
        self.patch_in = (_pad_cols(pe.weight, _ceil64(pe.weight.shape[1])), _bf16(pe.bias))
        self.action_in = (_pad_cols(ae.weight, _ceil64(ae.weight.shape[1])), _bf16(ae.bias))
        po, ao = model.proj_out, model.action_proj_out
        self.patch_out = _pad_rows(po.weight, po.bias, _ceil64(po.weight.shape[0])) + (po.weight.shape[0],)
        self.action_out = _pad_rows(ao.weight, ao.bias, _ceil64(ao.weight.shape[0])) + (ao.weight.shape[0],)
        self.emb = _Embedders(model.condition_embedder)
        self.emb_action = _Embedders(model.condition_embedder_action)
        self.text = None
        self._token_bufs = {}   # zero-padded input rows of action_tokens, by shape

    # -------------------------------------------------------------- pieces
    def embed_text(self, text_emb):
        """PixArtAlphaTextProjection (linear_1, tanh-GELU, linear_2), model.py:1078-1079."""
        B, T, C = text_emb.shape
        x = text_emb.reshape(B * T, C).to(torch.bfloat16).contiguous()
        h = ops.linear(x, *self.emb.x1, epilogue=_lib.EPI_GELU)
        return ops.linear(h, *self.emb.x2).reshape(B, T, self.dim)

    def prepare_context(self, text_emb):
        """Text projection + every layer's cross K/V, once per context."""
        self.text = self.embed_text(text_emb)
        self.stack.prepare_context(self.text)
        return self.text

    def embed_time(self, timesteps, repeat, action_mode):
        """(temb [B*L, D] fp32, timestep_proj [B, L, 6, D] bf16), model.py:1086-1093."""
        e = self.emb_action if action_mode else self.emb
        B, T = timesteps.shape
        n = B * T
        lib, st = _lib.load(), _lib.stream_ptr()
        t = timesteps.reshape(n).float().contiguous()
        feat = torch.empty(n, e.freq_dim, dtype=torch.bfloat16, device=t.device)
        _lib.check(lib.wamb_timestep_embedding(t.data_ptr(), n, e.freq_dim, feat.data_ptr(), st))
        h = ops.linear(feat, *e.t1, epilogue=_lib.EPI_SILU)
        temb = torch.empty(n, self.dim, dtype=torch.float32, device=t.device)
        ops.linear(h, *e.t2, out=temb)
        s = torch.empty(n, self.dim, dtype=torch.bfloat16, device=t.device)
        _lib.check(lib.wamb_silu(temb.data_ptr(), self.dim, 1, n, self.dim, s.data_ptr(), self.dim, st))
        proj = ops.linear(s, *e.tp)
        if repeat > 1:
            tr = torch.empty(n * repeat, self.dim, dtype=torch.float32, device=t.device)
            pr = torch.empty(n * repeat, 6 * self.dim, dtype=torch.bfloat16, device=t.device)
            _lib.check(lib.wamb_repeat_rows(temb.data_ptr(), n, self.dim * 4, repeat, tr.data_ptr(), st))
            _lib.check(lib.wamb_repeat_rows(proj.data_ptr(), n, 6 * self.dim * 2, repeat, pr.data_ptr(), st))
            temb, proj = tr, pr
        return temb, proj.reshape(B, T * repeat, 6, self.dim)

    # ------------------------------------------------------------- forward
    def forward(self, input_dict, update_cache=0, cache_name="pos", action_mode=False,
                candidate_cache_rows=None, context_rows=None):
        """input_dict as the reference's (noisy_latents [B, C, F, H, W],
        timesteps [B, F], text_emb or a prepared context, grid_id or
        rotary_emb). Action mode also takes action_tokens [B, L, C]
        (time-major, L = F H W) in place of noisy_latents, with
        action_grid = (F, H, W). context_rows ([B] int64): prepared-context
        row of each batch row (CFG rows over a [conditional, negative]
        context)."""
        if torch.is_grad_enabled():
            raise RuntimeError("NativeWanModel is inference-only; use no_grad/inference_mode")
        if candidate_cache_rows is not None and update_cache != 0:
            raise ValueError("candidate read-only forward requires inference and update_cache=0")
        lib, st = _lib.load(), _lib.stream_ptr()
        tokens = input_dict.get("action_tokens") if action_mode else None
        if tokens is not None:
            # Time-major action states: the input GEMM reads them through a
            # zero-padded copy (one row per token, the padding stays zero).
            if tokens.dim() != 3 or not tokens.is_cuda or tokens.dtype != torch.bfloat16:
                raise ValueError("action_tokens must be a CUDA bf16 [B, L, C] tensor")
            x = tokens.contiguous()
            B, L, C = x.shape
            Fr, H, W = input_dict["action_grid"]
            if Fr * H * W != L:
                raise ValueError("action_grid does not match the token count")
            w_in, b_in = self.action_in
            key = (B * L, w_in.shape[1])
            xa = self._token_bufs.get(key)
            if xa is None:
                xa = self._token_bufs[key] = torch.zeros(key, dtype=torch.bfloat16, device=x.device)
            _lib.check(lib.wamb_copy_cols(x.data_ptr(), C * 2, B * L, C * 2, xa.data_ptr(), w_in.shape[1] * 2, st))
            p1, p2, p3 = 1, 1, 1
        else:
            x = input_dict["noisy_latents"]
            if x.dim() != 5 or not x.is_cuda:
                raise ValueError("noisy_latents must be a CUDA [B, C, F, H, W] tensor")
            x = x.to(torch.bfloat16).contiguous()
            B, C, Fr, H, W = x.shape
            p1, p2, p3 = (1, 1, 1) if action_mode else self.patch_size
            L = (Fr // p1) * (H // p2) * (W // p3)
            w_in, b_in = self.action_in if action_mode else self.patch_in
            xa = torch.empty(B * L, w_in.shape[1], dtype=torch.bfloat16, device=x.device)
            _lib.check(lib.wamb_embed_gather(x.data_ptr(), B, C, Fr, H, W, p1, p2, p3, xa.data_ptr(),
                                             w_in.shape[1], st))
        h = ops.linear(xa, w_in, b_in).reshape(B, L, self.dim)
        ctx = None
        if self.text is None:
            ctx = self.embed_text(input_dict["text_emb"])
        rope = input_dict.get("rotary_emb")
        if rope is None:
            rope = rope_freqs(input_dict["grid_id"][0].to(device=x.device, dtype=torch.float64))
        ph, pw = (1, 1) if action_mode else (p2, p3)
        temb, tproj = self.embed_time(input_dict["timesteps"], (H // ph) * (W // pw), action_mode)
        h = self.stack.forward(h, ctx, tproj, rope, update_cache, cache_name, candidate_cache_rows,
                               context_rows=context_rows)
        n = torch.empty(B * L, self.dim, dtype=torch.bfloat16, device=x.device)
        _lib.check(lib.wamb_output_norm(h.data_ptr(), 0, B * L, self.dim, self.eps, self.table.data_ptr(),
                                        temb.data_ptr(), 1, L, L, n.data_ptr(), st))
        w_o, b_o, n_real = self.action_out if action_mode else self.patch_out
        y = ops.linear(n, w_o, b_o)
        if n_real != w_o.shape[0]:
            yr = torch.empty(B * L, n_real, dtype=torch.bfloat16, device=x.device)
            _lib.check(lib.wamb_copy_cols(y.data_ptr(), y.stride(0) * 2, B * L, n_real * 2, yr.data_ptr(),
                                          n_real * 2, st))
            y = yr
        if action_mode:
            return y.reshape(B, L, n_real)
        n_patch = p1 * p2 * p3
        return y.reshape(B, L * n_patch, n_real // n_patch)     # 'b l (n c) -> b (l n) c'

    __call__ = forward


class NativeActionDenoiser:
    """The action denoise loop of one chunk as one CUDA graph: `steps`
    updates, each a NativeWanModel forward in action mode with
    update_cache=0 (the KV history stays read-only) followed by the
    flow-match step of the sample in place (FastWAM runs 10 such updates per
    action chunk, fastwam-base/fullcode-v1/real_speculative.py:33,107). The
    context must be prepared first (NativeWanModel.prepare_context)."""

    def __init__(self, native_model, scheduler):
        self.nm, self.sched = native_model, scheduler
        self.graph, self.static = None, None

    def capture(self, noisy_latents, grid_id, steps=None, frames_per_step=None):
        """Record the chunk for inputs shaped like `noisy_latents`
        ([B, action_dim, F, H, W]); each update k uses the scheduler's
        timestep k for every frame."""
        nm, sc = self.nm, self.sched
        if nm.text is None:
            raise RuntimeError("prepare_context() first")
        steps = len(sc.timesteps) if steps is None else steps
        x = noisy_latents.to(torch.bfloat16).contiguous().clone()
        B, C, Fr, H, W = x.shape
        L = Fr * H * W
        ts = [torch.full((B, Fr), float(sc.timesteps[k]), device=x.device) for k in range(steps)]
        rope = rope_freqs(grid_id[0].to(device=x.device, dtype=torch.float64))   # once per chunk
        deltas = [sc.delta(sc.timesteps[k]) for k in range(steps)]
        lib = _lib.load()

        def chunk():
            for k in range(steps):
                v = nm.forward({"noisy_latents": x, "rotary_emb": rope, "timesteps": ts[k]}, 0, "pos", True)
                _lib.check(lib.wamb_flow_step_cl(x.data_ptr(), 0, v.data_ptr(), 0, B, C, L, deltas[k],
                                                 _lib.stream_ptr()))

        with torch.no_grad():
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            saved = x.clone()
            with torch.cuda.stream(s):
                chunk()                       # warm-up (allocations, first-use setup)
            torch.cuda.current_stream().wait_stream(s)
            x.copy_(saved)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                chunk()
        self.graph, self.static = g, {"x": x, "timesteps": ts, "steps": steps}
        return self.static

    def run(self, noisy_latents=None):
        """Denoise one chunk: copy new noise in (if given), replay, return the sample."""
        if self.graph is None:
            raise RuntimeError("capture() first")
        if noisy_latents is not None:
            self.static["x"].copy_(noisy_latents, non_blocking=True)
        self.graph.replay()
        return self.static["x"]

    def launches_per_chunk(self, with_cache=True):
        """Kernel launches of one chunk: per update the stack's launches plus
        gather, input GEMM, timestep features, 3 embedding GEMMs, SiLU,
        output norm, output GEMM and the step (= 10), + 2 row repeats when
        frames repeat over tokens, + 1 column copy for the 30-wide output."""
        return self.static["steps"] * (self.nm.stack.launches_per_step(with_cache) + 13)
