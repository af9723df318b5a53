"""NativeBlock: binds one block's parameters to the B200 block forward.

Mirrors the reference binding (算子研究/wam_ops/baseline/native.py:25-60 and
optimized/native.py:27-65): the 27 parameter tensors are read-only aliases
in the reference's fixed order, `__call__` takes the block's forward
arguments plus `debug`, and the whole forward is one call into libwamb.so
(`wamb_block_forward`); Python does no math on the hot path.
"""
import ctypes
import weakref

import torch

from . import _lib

_WORKSPACES = {}
_RETIRED = []   # outgrown workspaces, kept alive for the CUDA graphs that captured them


def workspace(device, nbytes):
    """One growing scratch buffer per device, shared by every block (blocks
    run one after another on the stream, so they can reuse it). A buffer that
    is outgrown is retired, never freed: a CUDA graph captured with it (e.g.
    the 1-row target forward of a speculative loop, captured before the
    7-row one grew the workspace) keeps a valid address. New buffers are
    zero-filled: the library keeps its stream-K flags (the first bytes of
    every layout) zero between calls."""
    key = torch.device(device).index if torch.device(device).index is not None else torch.cuda.current_device()
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _RETIRED.append(buf)
        buf = torch.zeros(max(nbytes, 1), dtype=torch.uint8, device=torch.device("cuda", key))
        _WORKSPACES[key] = buf
    return buf


def block_weights(block):
    """The 27 parameters in the reference order (baseline/native.py:31-46)."""
    table = block.scale_shift_table
    weights = [table]
    if hasattr(block.norm2, "weight") and block.norm2.weight is not None:
        weights += [block.norm2.weight, block.norm2.bias]
    else:
        empty = table.new_empty(0)
        weights += [empty, empty]
    for a in (block.attn1, block.attn2):
        for m in (a.to_q, a.to_k, a.to_v, a.to_out[0]):
            weights += [m.weight, m.bias]
        weights += [a.norm_q.weight, a.norm_k.weight]
    for m in (block.ffn.net[0].proj, block.ffn.net[2]):
        weights += [m.weight, m.bias]
    return [w.detach() for w in weights]


def block_eps(block):
    """eps order of the reference binding (baseline/native.py:50-52)."""
    norm2_eps = getattr(block.norm2, "eps", block.norm1.eps)
    return [block.norm1.eps, norm2_eps, block.norm3.eps, block.attn1.norm_q.eps,
            block.attn1.norm_k.eps, block.attn2.norm_q.eps, block.attn2.norm_k.eps]


def _check_weights(weights):
    dev = weights[3].device
    if dev.type != "cuda":
        raise RuntimeError("NativeBlock parameters must live on a CUDA device")
    out = []
    for i, t in enumerate(weights):
        if i in (1, 2) and t.numel() == 0:
            out.append(None)
            continue
        if t.device != dev:
            raise RuntimeError(f"frozen canonical parameter index {i} is on {t.device}, expected {dev}")
        if i <= 2:
            # modulation table and norm2 affine run in fp32 (the reference keeps
            # them fp32); a bf16 copy is widened once, exactly.
            if t.dtype not in (torch.float32, torch.bfloat16):
                raise RuntimeError(f"frozen canonical parameter index {i} dtype {t.dtype}")
            t = t.float().contiguous()
        else:
            if t.dtype != torch.bfloat16 or not t.is_contiguous():
                raise RuntimeError(f"frozen canonical parameter index {i} must be contiguous bf16, got {t.dtype}")
        out.append(t)
    return out


def quantize_weights_fp8(weights):
    """E4M3 copies of the eight step GEMM weights with per-output-channel
    fp32 scales (wamb_quantize_rows on each [N, K] weight), indexed like the
    27 reference parameters (None elsewhere)."""
    from .ops import quantize_rows
    w8, sc = [None] * 27, [None] * 27
    for i in _lib.FP8_WEIGHTS:
        w8[i], sc[i] = quantize_rows(weights[i])
    return w8, sc


class NativeBlock:
    """Bind the original parameter tensors; forward contains no Torch math ops."""

    def __init__(self, block, fused_ffn1=False, mode="sequential", fp8=False):
        if mode not in ("sequential", "tiled", "persistent"):
            raise ValueError("mode must be sequential, tiled or persistent")
        self.mode = mode
        self.fused_ffn1 = fused_ffn1
        self.block = weakref.ref(block)
        self.weights = _check_weights(block_weights(block))
        self.eps = block_eps(block)
        self.dim = block.attn1.to_q.weight.shape[1]
        self.heads = block.attn1.heads
        self.ffn_dim = block.ffn.net[0].proj.weight.shape[0]
        if self.dim != self.heads * 128:
            raise ValueError("the B200 block supports head_dim 128 only")
        self.fp8 = bool(fp8)
        self.w8, self.w8_scale = quantize_weights_fp8(self.weights) if self.fp8 else (None, None)

    # --------------------------------------------------------------- args
    def make_args(self, hidden_states, encoder_hidden_states, temb, rotary_emb, cache,
                  candidate_cache_rows, update_cache, out, cross_kv=None, context_rows=None,
                  keep=None, chained=False):
        keep = [] if keep is None else keep
        x = hidden_states
        if not (x.is_cuda and x.dtype in (torch.bfloat16, torch.float32) and x.is_contiguous()
                and x.dim() == 3):
            raise RuntimeError("hidden_states must be a contiguous CUDA bf16 (or fp32) [B, Q, D] tensor")
        B, Q, D = x.shape
        if D != self.dim:
            raise RuntimeError(f"hidden dim {D} != block dim {self.dim}")
        a = _lib.BlockArgs()
        a.batch, a.tokens, a.dim, a.heads, a.ffn_dim = B, Q, D, self.heads, self.ffn_dim
        for i, w in enumerate(self.weights):
            a.weights[i] = None if w is None else w.data_ptr()
        for i, e in enumerate(self.eps):
            a.eps[i] = float(e)
        a.x = x.data_ptr()
        a.x_is_f32 = int(x.dtype == torch.float32)
        if cross_kv is not None:
            k, v = cross_kv
            a.cross_k, a.cross_v = k.data_ptr(), v.data_ptr()
            a.context_batch = k.shape[0]
            a.context_tokens = k.shape[1]
        else:
            ctx = encoder_hidden_states
            if not (ctx.is_cuda and ctx.dtype == torch.bfloat16 and ctx.dim() == 3 and ctx.shape[2] == D):
                raise RuntimeError("encoder_hidden_states must be CUDA bf16 [Bc, C, D]")
            ctx = ctx.contiguous()
            keep.append(ctx)
            a.context = ctx.data_ptr()
            a.context_batch, a.context_tokens = ctx.shape[0], ctx.shape[1]
        if context_rows is not None:
            a.context_rows = context_rows.data_ptr()
        if temb.dim() != 4 or temb.shape[0] != B or temb.shape[2] != 6 or temb.shape[3] != D:
            raise RuntimeError("temb must be [B, L, 6, D]")
        if temb.dtype not in (torch.float32, torch.bfloat16):
            raise RuntimeError("temb must be fp32 or bf16")
        temb = temb.contiguous()
        keep.append(temb)
        a.temb, a.temb_len, a.temb_is_f32 = temb.data_ptr(), temb.shape[1], int(temb.dtype == torch.float32)
        if rotary_emb is not None:
            f = rotary_emb
            if f.dtype != torch.complex64:
                f = f.to(torch.complex64)
            f = f.reshape(f.shape[0], -1, f.shape[-1])
            if f.shape[1] != Q or f.shape[2] != 64:
                raise RuntimeError("rotary_emb must be complex [fb, Q, 1, 64]")
            f = torch.view_as_real(f.contiguous())
            keep.append(f)
            a.freq, a.freq_batch = f.data_ptr(), f.shape[0]
        if cache is not None:
            k, v, ids, mask, pred = (cache[n] for n in ("k", "v", "id", "mask", "is_pred"))
            if not (k.dtype == v.dtype == torch.bfloat16 and k.is_contiguous() and v.is_contiguous()
                    and k.shape == v.shape and k.dim() == 4 and k.shape[2] * k.shape[3] == D):
                raise RuntimeError("cache schema: K,V bf16 [Bp, pool, H, 128]")
            if not (ids.dtype == torch.int64 and mask.dtype == torch.bool and pred.dtype == torch.bool):
                raise RuntimeError("cache schema: id int64, mask/is_pred bool")
            a.cache_k, a.cache_v = k.data_ptr(), v.data_ptr()
            a.cache_id, a.cache_mask, a.cache_pred = ids.data_ptr(), mask.data_ptr(), pred.data_ptr()
            a.pool_batch, a.pool = k.shape[0], k.shape[1]
        if candidate_cache_rows is not None:
            r = candidate_cache_rows
            if r.ndim != 1 or r.numel() != B or r.dtype != torch.long or r.device != x.device:
                raise ValueError("invalid candidate_cache_rows for this KV cache")
            a.candidate_rows = r.data_ptr()
        a.update = int(update_cache)
        if self.fp8:
            a.fp8 = 1
            for i in _lib.FP8_WEIGHTS:
                a.w8[i], a.w8_scale[i] = self.w8[i].data_ptr(), self.w8_scale[i].data_ptr()
        if out.shape != x.shape or out.dtype not in (torch.bfloat16, torch.float32) or not out.is_contiguous():
            raise RuntimeError("out must be a contiguous bf16/fp32 tensor shaped like hidden_states")
        a.out = out.data_ptr()
        a.out_is_f32 = int(out.dtype == torch.float32)
        a.chained = int(bool(chained))
        return a

    def __call__(self, hidden_states, encoder_hidden_states, temb, rotary_emb,
                 update_cache=0, cache_name="pos", candidate_cache_rows=None, debug=False,
                 cross_kv=None, context_rows=None, out_dtype=None, out=None, chained=False):
        """Runs the block; returns hidden_states' dtype by default. out_dtype /
        out select an fp32 output (the residual stream without the final bf16
        rounding), which multi-layer stacks use between blocks. chained=True
        declares that the previous work on the current stream is a block call
        of the same shape (the previous layer of a stack), so that the KV
        bookkeeping may start beside its last GEMM."""
        if torch.is_grad_enabled():
            raise RuntimeError("NativeBlock is inference-only; use no_grad/inference_mode")
        block = self.block()
        caches = block.attn1.attn_caches or {}
        cache = caches.get(cache_name)
        if candidate_cache_rows is not None and (update_cache != 0 or cache is None):
            raise ValueError("candidate verification requires existing read-only KV")
        if out is None:
            out = torch.empty_like(hidden_states, dtype=out_dtype or hidden_states.dtype)
        keep = []
        a = self.make_args(hidden_states, encoder_hidden_states, temb, rotary_emb, cache,
                           candidate_cache_rows, update_cache, out, cross_kv, context_rows, keep,
                           chained)
        lib = _lib.load()
        nbytes = lib.wamb_block_workspace_bytes(a)
        ws = workspace(hidden_states.device, nbytes)
        a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
        _lib.check(lib.wamb_block_forward(a, _lib.stream_ptr()))
        if not debug:
            return out
        return self._taps(a, ws, out)

    def _taps(self, a, ws, out):
        offs = (ctypes.c_int64 * len(_lib.TAPS))()
        _lib.load().wamb_block_workspace_layout(a, offs)
        B, Q, D, F = a.batch, a.tokens, a.dim, a.ffn_dim
        M = B * Q
        C = a.context_batch * a.context_tokens
        shapes = {"qkv": (M, 3 * D), "gelu": (M, F), "cross_k": (C, D), "cross_v": (C, D)}
        result = {}
        if a.fp8:
            o8, os_ = offs[_lib.TAPS.index("a8")], offs[_lib.TAPS.index("a8_scale")]
            result["a8"] = ws[o8:o8 + M * max(D, F)].clone()  # last quantized GEMM input, raw E4M3
            result["a8_scale"] = ws[os_:os_ + 4 * M].view(torch.float32).clone()
        fp32 = ("residual1", "residual2")
        for i, name in enumerate(_lib.TAPS):
            o = offs[i]
            if o < 0:
                continue
            if name.startswith("a8"):
                continue
            if name.startswith("kv_"):
                n = {"kv_slots": Q, "kv_tiles": 2 * a.pool, "kv_counts": 2}[name]
                result[name] = ws[o:o + 4 * n].view(torch.int32).clone()
                continue
            shape = shapes.get(name, (M, D))
            n = shape[0] * shape[1]
            if name in fp32:
                result[name] = ws[o:o + 4 * n].view(torch.float32).view(shape).clone()
            else:
                result[name] = ws[o:o + 2 * n].view(torch.bfloat16).view(shape).clone()
        result["output"] = out
        return result
