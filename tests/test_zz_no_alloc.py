"""wamb_block_forward_noalloc against wamb_block_forward, through the C ABI.

Some callers cannot allocate device memory where they run a block: serving
loops that keep cudaMalloc / cudaFree (which can synchronise the device) off
their path, and hosts that reach the library through a thin FFI and own no
device allocator to hand it a workspace. They use the no-allocation entry
point, which takes no workspace and runs in a fixed scratch array inside the
library. Both entry points launch the same kernels on the same inputs, so
their results must agree bit for bit:

* two calls in a row with a KV cache (update_cache 0, then 1): the array
  keeps the previous call's contents, so the second call shows that nothing
  stale leaks into the output, the pool rows or the cache metadata;
* two no-allocation calls back to back on one stream with different
  workspace layouts (no cache, then a cache and a close row count), with no
  synchronisation between them: the second call's KV bookkeeping must not
  disturb the first call's buffers in the shared array;
* a call whose scratch need exceeds the array is refused with
  WAMB_ERR_WORKSPACE and launches nothing.

The file name sorts last so that a run stopping at the first failure has run
every other test first.
"""
import ctypes

import pytest
import torch

from blockutil import make_inputs, make_oracle_block, to_device_block
from wam_ops import _lib
from wam_ops.native import NativeBlock

pytestmark = pytest.mark.gpu


def _prefilled_cache(block, pool, heads, batch, seed):
    block.attn1.init_kv_cache("pos", pool, heads, 128, "cuda", torch.bfloat16, batch)
    c = block.attn1.attn_caches["pos"]
    g = torch.Generator(device="cuda").manual_seed(seed)
    c["k"].normal_(generator=g)
    c["v"].normal_(generator=g)
    c["mask"][:80] = True
    c["id"][:80] = torch.arange(80, device="cuda") // 40
    return c


def _device_inputs(B, Q, D, C, H, seed):
    x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=seed)
    return x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), r.cuda()


def _workspace_call(lib, native, x, ctx, temb, r, cache, update, keep):
    out = torch.empty_like(x)
    a = native.make_args(x, ctx, temb, r, cache, None, update, out, keep=keep)
    ws = torch.zeros(lib.wamb_block_workspace_bytes(a), dtype=torch.uint8, device="cuda")
    keep.append(ws)
    a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
    _lib.check(lib.wamb_block_forward(a, _lib.stream_ptr()))
    return out


def test_noalloc_matches_workspace_entry(cuda_device):
    D, H, F, B, Q, C, pool = 256, 2, 512, 2, 40, 24, 160
    blk = make_oracle_block(D, F, H, seed=77)
    ga, gb = to_device_block(blk), to_device_block(blk)
    ca = _prefilled_cache(ga, pool, H, B, seed=5)
    cb = _prefilled_cache(gb, pool, H, B, seed=5)
    na, nb = NativeBlock(ga), NativeBlock(gb)
    lib = _lib.load()
    stream = _lib.stream_ptr()
    with torch.no_grad():
        for call, update in enumerate((0, 1)):
            x, ctx, temb, r = _device_inputs(B, Q, D, C, H, seed=900 + call)
            keep = []
            out_ws = _workspace_call(lib, na, x, ctx, temb, r, ca, update, keep)

            out_na = torch.empty_like(x)
            b = nb.make_args(x, ctx, temb, r, cb, None, update, out_na, keep=keep)
            assert lib.wamb_block_workspace_bytes(b) <= _lib.NOALLOC_SCRATCH_BYTES
            _lib.check(lib.wamb_block_forward_noalloc(b, stream))
            torch.cuda.synchronize()
            assert _lib.device_status() == 0

            assert torch.equal(out_na, out_ws), (out_na.float() - out_ws.float()).abs().max().item()
            for name in ("id", "mask", "is_pred", "k", "v"):
                assert torch.equal(ca[name], cb[name]), name


def _layout(lib, a):
    offs = (ctypes.c_int64 * len(_lib.TAPS))()
    total = lib.wamb_block_workspace_layout(a, offs)
    return {name: offs[i] for i, name in enumerate(_lib.TAPS)}, total


def test_noalloc_back_to_back_layouts(cuda_device):
    """A no-cache call of 64 rows, then at once a cache call of fewer rows,
    both through the no-allocation entry point on one stream. The second
    call's KV scratch (slots, tiles, counts) lies inside the first call's
    residual / GELU buffers, which the first call's last GEMM reads: each
    output must still equal the workspace entry point's on the same inputs."""
    D, H, F, C, pool = 256, 2, 512, 24, 160
    blk = make_oracle_block(D, F, H, seed=79)
    lib = _lib.load()
    stream = _lib.stream_ptr()
    probe = NativeBlock(to_device_block(blk))
    x1 = torch.zeros(1, 64, D, dtype=torch.bfloat16, device="cuda")
    ctx0 = torch.zeros(1, C, D, dtype=torch.bfloat16, device="cuda")
    t0 = torch.zeros(1, 1, 6, D, device="cuda")
    l1, _ = _layout(lib, probe.make_args(x1, ctx0, t0, None, None, None, 0, x1))
    M1 = 64
    read_by_last_gemm = [(l1["residual2"], l1["residual2"] + 4 * M1 * D), (l1["gelu"], l1["gelu"] + 2 * M1 * F)]
    dummy = to_device_block(blk)
    cache = _prefilled_cache(dummy, pool, H, 1, seed=6)
    q2 = None
    for q in range(8, 64):
        xq = torch.zeros(1, q, D, dtype=torch.bfloat16, device="cuda")
        l2, _ = _layout(lib, probe.make_args(xq, ctx0, t0, None, cache, None, 0, xq))
        lo, hi = l2["kv_slots"], l2["kv_counts"] + 16
        if any(lo < b and a < hi for a, b in read_by_last_gemm):
            q2 = q
            break
    assert q2 is not None, "no row count puts the KV scratch over the first call's FFN2 inputs"
    shapes = ((1, 64, False), (1, q2, True))
    with torch.no_grad():
        ref_blocks = [to_device_block(blk) for _ in shapes]
        nat_blocks = [to_device_block(blk) for _ in shapes]
        inputs = [_device_inputs(B, Q, D, C, H, seed=950 + i) for i, (B, Q, _) in enumerate(shapes)]
        keep, refs = [], []
        for (B, Q, has_cache), g, inp in zip(shapes, ref_blocks, inputs):
            c = _prefilled_cache(g, pool, H, B, seed=6) if has_cache else None
            refs.append(_workspace_call(lib, NativeBlock(g), *inp, c, 0, keep))
        caches = [_prefilled_cache(g, pool, H, B, seed=6) if has_cache else None
                  for (B, Q, has_cache), g in zip(shapes, nat_blocks)]
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        outs = []
        for g, inp, c in zip(nat_blocks, inputs, caches):
            out = torch.empty_like(inp[0])
            a = NativeBlock(g).make_args(*inp, c, None, 0, out, keep=keep)
            _lib.check(lib.wamb_block_forward_noalloc(a, stream))
            outs.append(out)
        torch.cuda.synchronize()
        assert _lib.device_status() == 0
        for out, ref in zip(outs, refs):
            assert torch.equal(out, ref), (out.float() - ref.float()).abs().max().item()
        rc = ref_blocks[1].attn1.attn_caches["pos"]
        for name in ("id", "mask", "is_pred", "k", "v"):
            assert torch.equal(caches[1][name], rc[name]), name


def test_noalloc_rejects_calls_beyond_the_scratch(cuda_device):
    blk = make_oracle_block(256, 512, 2, seed=78)
    nb = NativeBlock(to_device_block(blk))
    B, Q, D = 1, 8192, 256   # ~46 MB of scratch at this shape
    x = torch.zeros(B, Q, D, dtype=torch.bfloat16, device="cuda")
    ctx = torch.zeros(B, 16, D, dtype=torch.bfloat16, device="cuda")
    temb = torch.zeros(B, 1, 6, D, device="cuda")
    out = torch.full_like(x, 7.0)
    lib = _lib.load()
    a = nb.make_args(x, ctx, temb, None, None, None, 0, out)
    assert lib.wamb_block_workspace_bytes(a) > _lib.NOALLOC_SCRATCH_BYTES
    assert lib.wamb_block_forward_noalloc(a, _lib.stream_ptr()) == 7  # WAMB_ERR_WORKSPACE
    assert b"no-allocation" in lib.wamb_last_error()
    torch.cuda.synchronize()
    assert bool((out == 7.0).all())   # nothing was launched
