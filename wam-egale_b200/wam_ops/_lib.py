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
        ("res", c_void_p), ("ldr", c_int64),
        ("table", c_void_p), ("temb", c_void_p), ("temb_is_f32", c_int32),
        ("temb_len", c_int32), ("rows_per_batch", c_int32), ("gate_index", c_int32),
        ("dim", c_int32),
    ]


EPI_BIAS, EPI_GELU, EPI_RES, EPI_RES_GATE = 0, 1, 2, 3

# Every symbol include/wamb.h declares; tests check the library exports them.
EXPORTED = (
    "wamb_last_error", "wamb_abi_version", "wamb_device_status", "wamb_linear",
)

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
