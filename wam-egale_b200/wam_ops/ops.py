"""Tensor-level wrappers over the C ABI (device tensors in, device tensors out).

These are the building blocks the block forward is made of, exposed for the
parity tests: each validates its tensors and calls one libwamb entry point
on the current CUDA stream.
"""
import torch

from . import _lib


def _bf16_2d(t, name):
    if not (t.is_cuda and t.dtype == torch.bfloat16):
        raise ValueError(f"{name} must be a CUDA bf16 tensor")
    if t.dim() != 2 or t.stride(1) != 1:
        raise ValueError(f"{name} must be 2-D with unit column stride")


_SK = {}


def sk_workspace(device):
    """Zero-filled stream-K scratch of wamb_linear on `device` (one per
    device; calls on one stream are ordered, so they share it)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _SK.get(idx)
    if buf is None:
        n = _lib.load().wamb_linear_sk_bytes()
        buf = _SK[idx] = torch.zeros(max(n, 1), dtype=torch.uint8, device=torch.device("cuda", idx))
    return buf


def linear(a, weights, biases=None, epilogue=_lib.EPI_BIAS, out=None, res=None,
           table=None, temb=None, rows_per_batch=None, gate_index=0, a_scale=None, w_scales=None):
    """out = epilogue(a @ cat(weights).T + cat(biases)) on the tcgen05 GEMM.

    `weights` is one [N, K] bf16 tensor or a list of up to three equally
    shaped ones whose outputs are concatenated along the columns (the QKV
    projection reads the three reference Linear weights in place).

    FP8: with `a` and the weights float8_e4m3fn, `a_scale` ([M] fp32 row
    scales) and `w_scales` (one [N] fp32 per weight) are required and the
    product is a_scale[m] * w_scale[n] * (a8 @ w8.T) (see quantize_rows).

    Small M: when the output tiles would leave SMs idle, K is split across
    the CTAs of a thread-block cluster (partials summed in split order in
    shared memory, so results do not depend on timing). M >= 512: the
    two-CTA kernel, with stream-K over every SM pair when the tiles leave
    the last round partly filled (scratch from sk_workspace()).
    """
    out_f32 = out is not None and out.dtype == torch.float32
    if isinstance(weights, torch.Tensor):
        weights = [weights]
    if biases is None or isinstance(biases, torch.Tensor):
        biases = [biases] * len(weights) if biases is None else [biases]
    fp8 = a.dtype == torch.float8_e4m3fn
    if isinstance(w_scales, torch.Tensor):
        w_scales = [w_scales]
    if fp8:
        if a.dim() != 2 or a.stride(1) != 1 or not a.is_cuda:
            raise ValueError("a must be a 2-D row-major CUDA tensor")
        if a_scale is None or w_scales is None or len(w_scales) != len(weights):
            raise ValueError("FP8 linear needs a_scale and one w_scale per weight")
        for t in [a_scale, *w_scales]:
            if t.dtype != torch.float32 or not t.is_contiguous():
                raise ValueError("FP8 scales must be contiguous fp32")
    else:
        _bf16_2d(a, "a")
    wdt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    n_g, k = weights[0].shape
    for w in weights:
        if w.shape != (n_g, k) or not w.is_contiguous() or w.dtype != wdt:
            raise ValueError(f"weights must be contiguous {wdt} [N, K] of equal shape")
    if a.shape[1] != k:
        raise ValueError("a and weight K differ")
    m = a.shape[0]
    n = n_g * len(weights)
    if out is None:
        out = torch.empty(m, n, device=a.device, dtype=torch.bfloat16)
    args = _lib.LinearArgs()
    args.a = a.data_ptr()
    args.lda = a.stride(0)
    args.m, args.k = m, k
    args.groups = len(weights)
    args.n_per_group = n_g
    for i, w in enumerate(weights):
        args.weight[i] = w.data_ptr()
        b = biases[i]
        args.bias[i] = None if b is None else b.data_ptr()
    args.out = out.data_ptr()
    args.ldo = out.stride(0)
    args.out_is_f32 = int(out_f32)
    args.epilogue = epilogue
    if m >= 512:
        sk = sk_workspace(a.device)
        args.sk_workspace, args.sk_workspace_bytes = sk.data_ptr(), sk.numel()
    if fp8:
        args.a_is_fp8 = 1
        args.a_scale = a_scale.data_ptr()
        for i, ws in enumerate(w_scales):
            args.w_scale[i] = ws.data_ptr()
    if res is not None:
        args.res = res.data_ptr()
        args.ldr = res.stride(0)
        args.res_is_f32 = int(res.dtype == torch.float32)
    if table is not None:
        args.table = table.data_ptr()
        args.temb = temb.data_ptr()
        args.temb_is_f32 = int(temb.dtype == torch.float32)
        args.temb_len = temb.shape[1]
        args.rows_per_batch = rows_per_batch
        args.gate_index = gate_index
        args.dim = n
    _lib.check(_lib.load().wamb_linear(args, _lib.stream_ptr()))
    return out


def quantize_rows(x, out=None, scale=None):
    """Row-wise E4M3 quantization on the GPU (wamb_quantize_rows): returns
    (q [M, K] float8_e4m3fn, scale [M] fp32) with scale = amax / 448 and
    q = e4m3(x * 448 / amax), amax = max(max |x[r]|, 1e-20). Used for
    activations (per token) and for weights (per output channel)."""
    if x.dim() != 2 or x.stride(1) != 1 or x.dtype not in (torch.bfloat16, torch.float32) or not x.is_cuda:
        raise ValueError("x must be a 2-D row-major bf16/fp32 CUDA tensor")
    m, k = x.shape
    if out is None:
        out = torch.empty(m, k, device=x.device, dtype=torch.float8_e4m3fn)
    if scale is None:
        scale = torch.empty(m, device=x.device, dtype=torch.float32)
    _lib.check(_lib.load().wamb_quantize_rows(
        x.data_ptr(), x.stride(0), int(x.dtype == torch.float32), m, k, out.data_ptr(), out.stride(0),
        scale.data_ptr(), _lib.stream_ptr()))
    return out, scale


def attention(q, k0, v0, *, heads, q_rows, q_col=0, k0_col=0, v0_col=0, src0_batch_stride,
              src0_len=None, tiles=None, n_tiles=None, src0_map=None, src0_broadcast=False,
              k1=None, v1=None, k1_col=0, v1_col=0, out=None, kv_splits=None):
    """Flash attention over 2-D row-major views (see wamb_attention_args).

    q: [batch*q_rows, ldq] bf16; k0/v0: [rows0, ld0] bf16; optional k1/v1:
    [batch*q_rows, ld1]. tiles: int32 [n, 2] (first row, length) with the
    count in the int32 device tensor n_tiles; otherwise src0_len rows.
    kv_splits: None (no split-key scratch), 0 (the library chooses) or a
    forced split factor; the scratch comes from a zero-filled per-device
    buffer. Returns out [batch*q_rows, heads*128] bf16.
    """
    for name, t in (("q", q), ("k0", k0), ("v0", v0)):
        _bf16_2d(t, name)
    batch = q.shape[0] // q_rows
    if out is None:
        out = torch.empty(batch * q_rows, heads * 128, device=q.device, dtype=torch.bfloat16)
    a = _lib.AttentionArgs()
    a.batch, a.heads, a.q_rows = batch, heads, q_rows
    a.q, a.ldq, a.q_total_rows, a.q_col = q.data_ptr(), q.stride(0), q.shape[0], q_col
    a.k0, a.v0, a.ld0, a.src0_total_rows = k0.data_ptr(), v0.data_ptr(), k0.stride(0), k0.shape[0]
    a.k0_col, a.v0_col = k0_col, v0_col
    a.src0_batch_stride = src0_batch_stride
    a.src0_map = None if src0_map is None else src0_map.data_ptr()
    a.src0_broadcast = int(src0_broadcast)
    if tiles is not None:
        a.tiles, a.n_tiles = tiles.data_ptr(), n_tiles.data_ptr()
    else:
        a.src0_len = src0_len
    if k1 is not None:
        a.k1, a.v1, a.ld1, a.k1_col, a.v1_col = k1.data_ptr(), v1.data_ptr(), k1.stride(0), k1_col, v1_col
    a.out, a.ldo = out.data_ptr(), out.stride(0)
    lib = _lib.load()
    if kv_splits is not None:
        a.kv_splits = kv_splits
        need = lib.wamb_attention_split_bytes(a)
        if need:
            buf = _split_workspace(q.device, need)
            a.split_workspace, a.split_workspace_bytes = buf.data_ptr(), buf.numel()
    _lib.check(lib.wamb_attention(a, _lib.stream_ptr()))
    return out


_SPLIT = {}


def _split_workspace(device, nbytes):
    """Zero-filled split-key scratch of wamb_attention (one growing buffer
    per device; outgrown buffers are kept, as captured graphs may use them)."""
    idx = device.index if device.index is not None else torch.cuda.current_device()
    buf = _SPLIT.get(idx)
    if buf is None or buf.numel() < nbytes:
        if buf is not None:
            _SPLIT.setdefault("retired", []).append(buf)
        buf = _SPLIT[idx] = torch.zeros(nbytes, dtype=torch.uint8, device=torch.device("cuda", idx))
    return buf


def sdpa(q, k, v):
    """The reference's `sdpa(q, k, v)` contract: contiguous bf16 [B, S, H, 128]
    (算子研究/wam_ops/optimized/csrc/attention.cu:121-181); returns [B, Sq, H, 128]."""
    B, Sq, H, d = q.shape
    Sk = k.shape[1]
    if d != 128 or k.shape != v.shape or k.shape[0] != B or k.shape[2] != H:
        raise ValueError("expected q [B,Sq,H,128], k = v [B,Sk,H,128]")
    if not (q.is_contiguous() and k.is_contiguous() and v.is_contiguous()):
        raise ValueError("Q/K/V must be contiguous; no hidden copies")
    out = attention(q.view(B * Sq, H * d), k.view(B * Sk, H * d), v.view(B * Sk, H * d), heads=H,
                    q_rows=Sq, src0_batch_stride=Sk, src0_len=Sk)
    return out.view(B, Sq, H, d)
