"""CPU checks of the C ABI: the library loads, exports every entry point
include/wamb.h declares, reports its version, computes workspace layouts and
rejects bad arguments on the host without touching a GPU."""
import ctypes
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from wam_ops import _lib

HEADER = Path(__file__).resolve().parents[1] / "include" / "wamb.h"


def test_header_symbols_exported():
    lib = _lib.load()
    declared = set(re.findall(r"WAMB_API\s+[\w\s\*]+?\b(wamb_\w+)\s*\(", HEADER.read_text()))
    assert declared == set(_lib.EXPORTED)
    for name in declared:
        assert hasattr(lib, name), name
    assert lib.wamb_abi_version() == _lib.ABI_VERSION


@pytest.mark.parametrize("cname,pyname", [("wamb_linear_args", "LinearArgs"),
                                            ("wamb_attention_args", "AttentionArgs"),
                                            ("wamb_block_args", "BlockArgs"),
                                            ("wamb_draft_params", "DraftParams")])
def test_struct_layout_matches_header(tmp_path, cname, pyname):
    """Every field offset of the ctypes mirror equals the C compiler's."""
    cc = shutil.which("gcc") or shutil.which("cc")
    if cc is None:
        pytest.skip("no C compiler")
    st = getattr(_lib, pyname)
    lines = [f'printf("%zu\\n", sizeof({cname}));']
    lines += [f'printf("%zu\\n", offsetof({cname}, {f[0]}));' for f in st._fields_]
    src = tmp_path / "probe.c"
    src.write_text("#include <stdio.h>\n#include <stddef.h>\n#include \"wamb.h\"\nint main(void){"
                   + "".join(lines) + "return 0;}\n")
    exe = tmp_path / "probe"
    subprocess.run([cc, "-I", str(HEADER.parent), str(src), "-o", str(exe)], check=True)
    got = [int(v) for v in subprocess.run([str(exe)], capture_output=True, text=True,
                                          check=True).stdout.split()]
    want = [ctypes.sizeof(st)] + [getattr(st, f[0]).offset for f in st._fields_]
    assert got == want


def _args(**kw):
    a = _lib.BlockArgs()
    a.batch, a.tokens, a.dim, a.heads, a.ffn_dim = 1, 48, 256, 2, 512
    a.context_tokens, a.context_batch = 32, 1
    for k, v in kw.items():
        setattr(a, k, v)
    return a


def test_workspace_layout():
    lib = _lib.load()
    a = _args()
    offs = (ctypes.c_int64 * len(_lib.TAPS))()
    total = lib.wamb_block_workspace_layout(a, offs)
    assert total == lib.wamb_block_workspace_bytes(a)
    M, D, F = 48, 256, 512
    assert offs[_lib.TAPS.index("sk_flags")] == 0           # stream-K flags first in every layout
    assert offs[_lib.TAPS.index("modulated1")] == 16384         # after the 16 KB zero region
    assert offs[_lib.TAPS.index("sk_part")] == -1           # M < 512: no two-CTA GEMM
    assert offs[_lib.TAPS.index("kv_slots")] == -1          # no cache
    assert offs[_lib.TAPS.index("norm2")] >= 0
    assert total >= (12 * M * D + M * F) * 2                # residual stream taps are fp32
    assert all(o % 256 == 0 for o in offs if o >= 0)
    assert offs[_lib.TAPS.index("a8")] == -1                # bf16 path


def test_workspace_layout_fp8():
    """FP8 path: no bf16 LayerNorm outputs, one E4M3 buffer of M x max(D, F)
    bytes and M fp32 row scales instead."""
    lib = _lib.load()
    a = _args(fp8=1)
    offs = (ctypes.c_int64 * len(_lib.TAPS))()
    total = lib.wamb_block_workspace_layout(a, offs)
    M, F = 48, 512
    for t in ("modulated1", "norm2", "modulated3"):
        assert offs[_lib.TAPS.index(t)] == -1
    a8, sc = offs[_lib.TAPS.index("a8")], offs[_lib.TAPS.index("a8_scale")]
    assert a8 >= 0 and sc >= a8 + M * F and total >= sc + 4 * M


def test_fp8_block_requires_e4m3_weights():
    lib = _lib.load()
    a = _args(fp8=1)
    assert lib.wamb_block_forward(a, None) != 0
    assert lib.wamb_last_error()


def test_quantize_rows_rejects_bad_args():
    lib = _lib.load()
    assert lib.wamb_quantize_rows(None, 8, 0, 4, 8, None, 16, None, None) != 0   # null pointers
    assert lib.wamb_quantize_rows(None, 8, 0, 4, 12, None, 16, None, None) == 2  # k % 8


@pytest.mark.parametrize("kw,code", [
    ({"dim": 250}, 2),               # dim must be heads * 128
    ({"tokens": 0}, 2),
    ({"update": 3}, 1),
])
def test_block_forward_rejects_bad_args(kw, code):
    lib = _lib.load()
    a = _args(**kw)
    rc = lib.wamb_block_forward(a, None)
    assert rc != 0
    assert lib.wamb_last_error()


def test_cross_kv_rejects_bad_args():
    """wamb_cross_kv checks its buffers on the host before any launch: a
    missing context or output (1), K and V outputs that are one buffer (1,
    its two-group launch would write both into it), unaligned outputs (3)."""
    lib = _lib.load()
    lib.wamb_cross_kv.argtypes = [ctypes.POINTER(_lib.BlockArgs), ctypes.c_void_p, ctypes.c_void_p,
                                  ctypes.c_void_p]
    a = _args()
    assert lib.wamb_cross_kv(a, 0x1000, 0x2000, None) == 1        # no context
    a.context = 0x3000
    assert lib.wamb_cross_kv(a, None, 0x2000, None) == 1
    assert lib.wamb_cross_kv(a, 0x1000, 0x1000, None) == 1        # K and V in one buffer
    assert lib.wamb_cross_kv(a, 0x1008, 0x2000, None) == 3        # K not 16-byte aligned
    assert lib.wamb_last_error()


def test_linear_rejects_bad_shapes():
    lib = _lib.load()
    a = _lib.LinearArgs()
    a.m, a.k, a.groups, a.n_per_group = 10, 100, 1, 64     # K not a multiple of 64
    assert lib.wamb_linear(a, None) == 2
    a.k, a.groups = 128, 4
    assert lib.wamb_linear(a, None) == 1
    a.k, a.groups, a.a_is_fp8 = 192, 1, 1                 # E4M3 K must be a multiple of 128
    assert lib.wamb_linear(a, None) == 2


def test_workspace_layout_is_the_taps():
    """Below 512 rows the workspace holds the named intermediates and the
    stream-K flags only (small-M GEMMs reduce their split-K partials in
    cluster shared memory, not in the workspace): the last tap ends the
    layout, and a 224-row D 3072 verify batch fits the no-allocation entry
    point's fixed scratch."""
    lib = _lib.load()
    offs = (ctypes.c_int64 * len(_lib.TAPS))()
    small = _args(batch=7, tokens=32, dim=3072, heads=24, ffn_dim=14336)
    total = lib.wamb_block_workspace_layout(small, offs)
    assert lib.wamb_block_workspace_bytes(small) == total
    gelu = offs[_lib.TAPS.index("gelu")]
    assert gelu == max(o for o in offs if o >= 0)          # no cache, bf16: GELU output is last
    assert total == (gelu + 7 * 32 * 14336 * 2 + 255) // 256 * 256
    assert total <= _lib.NOALLOC_SCRATCH_BYTES
