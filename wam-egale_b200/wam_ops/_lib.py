"""ctypes binding of libwamb.so (the C ABI in include/wamb.h).

The library is the only compute path: there is no PyTorch or CPU fallback.
If the shared object is missing, or the process has no sm_100 GPU, every
entry point raises instead of computing something else.
"""
import ctypes
import os
from pathlib import Path

_HERE = Path(__file__).resolve().parent
LIB_PATH = _HERE.parent / "lib" / "libwamb.so"

c_void_p = ctypes.c_void_p
c_int32 = ctypes.c_int32
c_int64 = ctypes.c_int64


class LinearArgs(ctypes.Structure):
    """Mirror of `wamb_linear_args` (include/wamb.h)."""
    _fields_ = [
        ("a", c_void_p), ("lda", c_int64), ("m", c_int32), ("k", c_int32),
        ("groups", c_int32), ("n_per_group", c_int32),
        ("weight", c_void_p * 3), ("bias", c_void_p * 3),
        ("out", c_void_p), ("ldo", c_int64), ("epilogue", c_int32),
        ("res", c_void_p), ("ldr", c_int64), ("res_is_f32", c_int32), ("out_is_f32", c_int32),
        ("table", c_void_p), ("temb", c_void_p), ("temb_is_f32", c_int32),
        ("temb_len", c_int32), ("rows_per_batch", c_int32), ("gate_index", c_int32),
        ("dim", c_int32),
        ("a_is_fp8", c_int32), ("a_scale", c_void_p), ("w_scale", c_void_p * 3),
        ("sk_workspace", c_void_p), ("sk_workspace_bytes", ctypes.c_size_t),
    ]


EPI_BIAS, EPI_GELU, EPI_RES, EPI_RES_GATE, EPI_SILU = 0, 1, 2, 3, 4


class AttentionArgs(ctypes.Structure):
    """Mirror of `wamb_attention_args` (include/wamb.h)."""
    _fields_ = [
        ("batch", c_int32), ("heads", c_int32), ("q_rows", c_int32),
        ("q", c_void_p), ("ldq", c_int64), ("q_total_rows", c_int64), ("q_col", c_int32),
        ("k0", c_void_p), ("v0", c_void_p), ("ld0", c_int64), ("src0_total_rows", c_int64),
        ("k0_col", c_int32), ("v0_col", c_int32),
        ("src0_batch_stride", c_int32),
        ("src0_map", c_void_p),
        ("src0_broadcast", c_int32),
        ("tiles", c_void_p), ("n_tiles", c_void_p),
        ("src0_len", c_int32),
        ("k1", c_void_p), ("v1", c_void_p), ("ld1", c_int64), ("k1_col", c_int32), ("v1_col", c_int32),
        ("out", c_void_p), ("ldo", c_int64),
        ("split_workspace", c_void_p), ("split_workspace_bytes", ctypes.c_size_t), ("kv_splits", c_int32),
    ]


class DraftParams(ctypes.Structure):
    """Mirror of `wamb_draft_params` (include/wamb.h)."""
    _fields_ = [
        ("tokens", c_int32), ("channels", c_int32), ("width", c_int32), ("heads", c_int32), ("ffn", c_int32),
        ("ln_eps", ctypes.c_float),
        ("embed_w", c_void_p), ("embed_b", c_void_p), ("position", c_void_p),
        ("in_proj_w", c_void_p), ("in_proj_b", c_void_p), ("out_proj_w", c_void_p), ("out_proj_b", c_void_p),
        ("linear1_w", c_void_p), ("linear1_b", c_void_p), ("linear2_w", c_void_p), ("linear2_b", c_void_p),
        ("norm1_w", c_void_p), ("norm1_b", c_void_p), ("norm2_w", c_void_p), ("norm2_b", c_void_p),
        ("head_w", c_void_p), ("head_b", c_void_p),
        ("feature_mean", c_void_p), ("feature_std", c_void_p),
        ("residual_mean", c_void_p), ("residual_std", c_void_p),
    ]


class BlockArgs(ctypes.Structure):
    """Mirror of `wamb_block_args` (include/wamb.h)."""
    _fields_ = [
        ("batch", c_int32), ("tokens", c_int32), ("dim", c_int32), ("heads", c_int32),
        ("ffn_dim", c_int32),
        ("context_tokens", c_int32), ("context_batch", c_int32),
        ("weights", c_void_p * 27),
        ("eps", ctypes.c_double * 7),
        ("x", c_void_p), ("x_is_f32", c_int32), ("out_is_f32", c_int32),
        ("context", c_void_p), ("cross_k", c_void_p), ("cross_v", c_void_p),
        ("context_rows", c_void_p),
        ("temb", c_void_p), ("temb_len", c_int32), ("temb_is_f32", c_int32),
        ("freq", c_void_p), ("freq_batch", c_int32),
        ("cache_k", c_void_p), ("cache_v", c_void_p), ("cache_id", c_void_p),
        ("cache_mask", c_void_p), ("cache_pred", c_void_p),
        ("pool", c_int32), ("pool_batch", c_int32),
        ("candidate_rows", c_void_p),
        ("update", c_int32),
        ("out", c_void_p),
        ("workspace", c_void_p), ("workspace_bytes", ctypes.c_size_t),
        ("fp8", c_int32), ("w8", c_void_p * 27), ("w8_scale", c_void_p * 27),
        ("chained", c_int32),
    ]


# Workspace taps (enum wamb_tap).
TAPS = ("modulated1", "qkv", "self_attention", "residual1", "norm2", "cross_q", "cross_k",
        "cross_v", "cross_attention", "residual2", "modulated3", "gelu", "kv_slots",
        "kv_tiles", "kv_counts", "a8", "a8_scale", "sk_flags", "sk_part", "attn_part")

# Weight slots the FP8 path reads as E4M3 (self q/k/v/out, cross q/out, FFN).
FP8_WEIGHTS = (3, 5, 7, 9, 13, 19, 23, 25)

ABI_VERSION = 107

# Every symbol include/wamb.h declares; tests check the library exports them.
EXPORTED = (
    "wamb_last_error", "wamb_abi_version", "wamb_device_status", "wamb_linear", "wamb_linear_sk_bytes",
    "wamb_attention", "wamb_attention_split_bytes", "wamb_block_workspace_bytes", "wamb_block_workspace_layout",
    "wamb_block_forward", "wamb_cross_kv", "wamb_block_forward_noalloc", "wamb_quantize_rows",
    "wamb_timestep_embedding", "wamb_silu", "wamb_embed_gather", "wamb_output_norm", "wamb_copy_cols",
    "wamb_flow_step", "wamb_repeat_rows", "wamb_flow_step_cl",
    "wamb_draft_forward", "wamb_spec_scores", "wamb_spec_route", "wamb_spec_expand", "wamb_spec_commit",
    "wamb_cfg_combine",
)

# Size of the fixed scratch array behind wamb_block_forward_noalloc.
NOALLOC_SCRATCH_BYTES = 32 << 20

_lib = None


class WambError(RuntimeError):
    """Raised when a libwamb call returns a non-zero status."""


def load():
    """Load libwamb.so once; raise if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise WambError(f"{LIB_PATH} is missing: run __graft_entry__.build() (no fallback path exists)")
    lib = ctypes.CDLL(str(LIB_PATH))
    lib.wamb_last_error.restype = ctypes.c_char_p
    lib.wamb_abi_version.restype = c_int32
    lib.wamb_device_status.argtypes = [c_void_p, ctypes.POINTER(c_int32)]
    lib.wamb_linear.argtypes = [ctypes.POINTER(LinearArgs), c_void_p]
    lib.wamb_linear_sk_bytes.restype = ctypes.c_size_t
    lib.wamb_attention.argtypes = [ctypes.POINTER(AttentionArgs), c_void_p]
    lib.wamb_attention_split_bytes.argtypes = [ctypes.POINTER(AttentionArgs)]
    lib.wamb_attention_split_bytes.restype = ctypes.c_size_t
    lib.wamb_block_workspace_bytes.argtypes = [ctypes.POINTER(BlockArgs)]
    lib.wamb_block_workspace_bytes.restype = ctypes.c_size_t
    lib.wamb_block_workspace_layout.argtypes = [ctypes.POINTER(BlockArgs), ctypes.POINTER(c_int64)]
    lib.wamb_block_workspace_layout.restype = ctypes.c_size_t
    lib.wamb_block_forward.argtypes = [ctypes.POINTER(BlockArgs), c_void_p]
    lib.wamb_cross_kv.argtypes = [ctypes.POINTER(BlockArgs), c_void_p, c_void_p, c_void_p]
    lib.wamb_block_forward_noalloc.argtypes = [ctypes.POINTER(BlockArgs), c_void_p]
    lib.wamb_quantize_rows.argtypes = [c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p, c_int64,
                                       c_void_p, c_void_p]
    lib.wamb_timestep_embedding.argtypes = [c_void_p, c_int32, c_int32, c_void_p, c_void_p]
    lib.wamb_silu.argtypes = [c_void_p, c_int64, c_int32, c_int32, c_int32, c_void_p, c_int64, c_void_p]
    lib.wamb_embed_gather.argtypes = [c_void_p] + [c_int32] * 8 + [c_void_p, c_int32, c_void_p]
    lib.wamb_output_norm.argtypes = [c_void_p, c_int32, c_int32, c_int32, ctypes.c_double, c_void_p, c_void_p,
                                     c_int32, c_int32, c_int32, c_void_p, c_void_p]
    lib.wamb_copy_cols.argtypes = [c_void_p, c_int64, c_int32, c_int32, c_void_p, c_int64, c_void_p]
    lib.wamb_flow_step_cl.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int32, c_int32, c_int64,
                                      ctypes.c_float, c_void_p]
    lib.wamb_repeat_rows.argtypes = [c_void_p, c_int32, c_int32, c_int32, c_void_p, c_void_p]
    lib.wamb_flow_step.argtypes = [c_void_p, c_int32, c_void_p, c_int32, c_int64, ctypes.c_float, c_void_p]
    lib.wamb_draft_forward.argtypes = [ctypes.POINTER(DraftParams), c_void_p, c_void_p, c_int32, c_void_p, c_int32,
                                       c_void_p, c_void_p]
    lib.wamb_spec_scores.argtypes = [c_void_p, c_void_p, c_int32, c_int64, c_int32, ctypes.POINTER(c_int32),
                                     ctypes.POINTER(c_int32), ctypes.POINTER(ctypes.c_float), c_int32, c_void_p,
                                     c_void_p]
    lib.wamb_spec_route.argtypes = [c_void_p, c_int32, ctypes.c_double, c_void_p, c_void_p]
    lib.wamb_spec_expand.argtypes = [c_void_p, c_void_p, c_int32, c_int32, c_int32, c_int64, ctypes.c_float,
                                     c_void_p, c_void_p]
    lib.wamb_spec_commit.argtypes = [c_void_p, c_void_p, c_void_p, c_int32, c_int64, ctypes.c_float,
                                     ctypes.c_float, ctypes.c_float, c_void_p, c_void_p, c_void_p]
    lib.wamb_cfg_combine.argtypes = [c_void_p, c_void_p, c_int32, c_int64, ctypes.c_float, c_void_p, c_void_p]
    if lib.wamb_abi_version() != ABI_VERSION:
        raise WambError(f"{LIB_PATH} has ABI {lib.wamb_abi_version()}, expected {ABI_VERSION}: rebuild")
    _lib = lib
    return lib


def check(rc):
    if rc != 0:
        msg = load().wamb_last_error().decode(errors="replace")
        raise WambError(f"libwamb error {rc}: {msg}")


def stream_ptr(stream=None):
    import torch
    s = torch.cuda.current_stream() if stream is None else stream
    return c_void_p(s.cuda_stream)


def device_status(stream=None):
    """Synchronise the stream and return (and clear) the device error word."""
    code = c_int32(0)
    check(load().wamb_device_status(stream_ptr(stream), ctypes.byref(code)))
    return code.value


def ptr(t):
    return None if t is None else c_void_p(t.data_ptr())
