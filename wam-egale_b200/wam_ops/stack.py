"""NativeStack: the 30-block denoise step of WanTransformer3DModel
(model.py:1091-1098) on the B200 block, optionally as one CUDA graph.

Each layer is a WholeLayerBlock with its cross-attention K/V prepared once
per context (whole_layer.py). Between layers the residual stream stays fp32
(the block's x_is_f32 / out_is_f32 mode): the first layer reads the caller's
bf16 hidden states and the last layer writes bf16, so the stack rounds the
residual stream once instead of once per layer. All layers share one
workspace, so a step allocates nothing after the first call, and
`capture()` records the whole step (420 kernel launches at 30 layers) in a
CUDA graph that `replay()` launches with one call.
"""
import torch

from . import _lib
from .whole_layer import WholeLayerBlock, prepared_context


class NativeStack:
    def __init__(self, blocks, fp8=False):
        """fp8=True runs the step's GEMMs on E4M3 weights (per-output-channel
        scales) and per-token E4M3 activations (the block's fp8 mode)."""
        self.fp8 = bool(fp8)
        self.layers = [WholeLayerBlock(b, fp8=fp8) for b in blocks]
        self.graph = None
        self._static = None

    def prepare_context(self, context):
        """Cross K/V of every layer for this context (outside timed regions)."""
        with torch.no_grad():
            rows, roots, compact = prepared_context(context)
            kv = torch.empty(len(self.layers), 2, *compact.shape, dtype=torch.bfloat16, device=compact.device)
            for layer, kv_l in zip(self.layers, kv):
                layer.set_context(rows, roots, compact, kv_l)

    def forward(self, hidden_states, encoder_hidden_states, temb, rotary_emb, update_cache=0,
                cache_name="pos", candidate_cache_rows=None, out=None, context_rows=None):
        """One denoise step through every layer; returns bf16 [B, Q, D].
        context_rows: per-call prepared-context row of each batch row."""
        if torch.is_grad_enabled():
            raise RuntimeError("NativeStack is inference-only; use no_grad/inference_mode")
        B, Q, D = hidden_states.shape
        dev = hidden_states.device
        bufs = [torch.empty(B, Q, D, dtype=torch.float32, device=dev) for _ in range(2)]
        h = hidden_states
        n = len(self.layers)
        for i, layer in enumerate(self.layers):
            last = i == n - 1
            dst = (out if out is not None else torch.empty(B, Q, D, dtype=torch.bfloat16, device=dev)) \
                if last else bufs[i % 2]
            # Layers after the first follow a block call of the same shape on
            # this stream, so their KV bookkeeping may start beside its last GEMM.
            layer(h, encoder_hidden_states, temb, rotary_emb, update_cache, cache_name,
                  candidate_cache_rows, out=dst, context_rows=context_rows, chained=i > 0)
            h = dst
        return h

    __call__ = forward

    def capture(self, hidden_states, encoder_hidden_states, temb, rotary_emb, update_cache=0,
                cache_name="pos", candidate_cache_rows=None, warmup=1):
        """Record one step as a CUDA graph over static copies of the inputs.
        update_cache must leave the cache ready for the next replay
        (update 0 restores the mask, so repeated denoise steps are stable)."""
        if update_cache != 0:
            raise ValueError("graph capture is for repeated denoise steps (update_cache=0)")
        static = {
            "x": hidden_states.clone(), "temb": temb.clone(),
            "rope": None if rotary_emb is None else rotary_emb.clone(),
            "rows": None if candidate_cache_rows is None else candidate_cache_rows.clone(),
        }
        static["out"] = torch.empty_like(static["x"], dtype=torch.bfloat16)
        args = (static["x"], encoder_hidden_states, static["temb"], static["rope"], 0, cache_name,
                static["rows"])
        with torch.no_grad():
            s = torch.cuda.Stream()
            s.wait_stream(torch.cuda.current_stream())
            with torch.cuda.stream(s):
                for _ in range(warmup):
                    self.forward(*args, out=static["out"])
            torch.cuda.current_stream().wait_stream(s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g):
                self.forward(*args, out=static["out"])
        self.graph, self._static = g, static
        return static

    def replay(self, hidden_states=None, temb=None):
        """Copy new inputs into the captured buffers (if given) and replay."""
        if self.graph is None:
            raise RuntimeError("capture() first")
        if hidden_states is not None:
            self._static["x"].copy_(hidden_states, non_blocking=True)
        if temb is not None:
            self._static["temb"].copy_(temb, non_blocking=True)
        self.graph.replay()
        return self._static["out"]

    @staticmethod
    def launches_per_layer(with_cache, fp8, cross_prepared=True):
        """Kernel launches of one layer (see launches_per_step)."""
        return 13 + (1 if with_cache else 0) + (0 if cross_prepared else 3) + (3 if fp8 else 0)

    def launches_per_step(self, with_cache, cross_prepared=True):
        """Kernel launches of one step (the count bench.py reports): per layer
        LN1, QKV, RMS+RoPE, attention, O, LN2, cross-Q, RMS, cross attention,
        cross-O, LN3, FFN1, FFN2 = 13, + KV layout with a cache, + 3 when the
        cross K/V is computed per call, + 3 row-quantize passes (self and cross
        attention output, GELU output) in fp8 mode."""
        return self.launches_per_layer(with_cache, self.fp8, cross_prepared) * len(self.layers)


def device_error():
    """Synchronise and return the device error word (0 = ok)."""
    return _lib.device_status()
