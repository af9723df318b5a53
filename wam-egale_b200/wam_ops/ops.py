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


def linear(a, weights, biases=None, epilogue=_lib.EPI_BIAS, out=None, res=None,
           table=None, temb=None, rows_per_batch=None, gate_index=0):
    """out = epilogue(a @ cat(weights).T + cat(biases)) on the tcgen05 GEMM.

    `weights` is one [N, K] bf16 tensor or a list of up to three equally
    shaped ones whose outputs are concatenated along the columns (the QKV
    projection reads the three reference Linear weights in place).
    """
    if isinstance(weights, torch.Tensor):
        weights = [weights]
    if biases is None or isinstance(biases, torch.Tensor):
        biases = [biases] * len(weights) if biases is None else [biases]
    _bf16_2d(a, "a")
    n_g, k = weights[0].shape
    for w in weights:
        if w.shape != (n_g, k) or not w.is_contiguous() or w.dtype != torch.bfloat16:
            raise ValueError("weights must be contiguous bf16 [N, K] of equal shape")
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
    args.epilogue = epilogue
    if res is not None:
        args.res = res.data_ptr()
        args.ldr = res.stride(0)
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
