"""wamb_block_forward_noalloc against wamb_block_forward, through the C ABI.

Callers that cannot allocate device memory where they run a block (work
recorded into a CUDA graph, serving loops that keep the device allocator off
their path, hosts that reach the library through a thin FFI) use the
no-allocation entry point: it takes no workspace and runs in a fixed scratch
array inside the library. This file checks that it computes what the
workspace entry point computes, on two calls in a row (the array keeps the
previous call's contents, so the second call shows nothing stale leaks), with
the same KV-cache effects, and that it refuses a call whose scratch need
exceeds the array. Tolerance: the block parity gate of tests/blockutil.py
(cos >= 0.9999, max |err| <= 2e-2), here against the workspace entry point's
output. The file name sorts last so that a run stopping at the first failure
has run every other test first.
"""
import pytest
import torch

from blockutil import assert_parity, make_inputs, make_oracle_block, to_device_block
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
            x, ctx, temb, r = make_inputs(B, Q, D, C, H, seed=900 + call)
            x, ctx, temb, r = x.cuda().bfloat16(), ctx.cuda().bfloat16(), temb.cuda(), r.cuda()
            keep = []
            out_ws = torch.empty_like(x)
            a = na.make_args(x, ctx, temb, r, ca, None, update, out_ws, keep=keep)
            ws = torch.empty(lib.wamb_block_workspace_bytes(a), dtype=torch.uint8, device="cuda")
            a.workspace, a.workspace_bytes = ws.data_ptr(), ws.numel()
            _lib.check(lib.wamb_block_forward(a, stream))

            out_na = torch.empty_like(x)
            b = nb.make_args(x, ctx, temb, r, cb, None, update, out_na, keep=keep)
            assert lib.wamb_block_workspace_bytes(b) <= _lib.NOALLOC_SCRATCH_BYTES
            _lib.check(lib.wamb_block_forward_noalloc(b, stream))
            torch.cuda.synchronize()
            assert _lib.device_status() == 0

            assert_parity(out_na, out_ws.float())
            for name in ("id", "mask", "is_pred"):
                assert torch.equal(ca[name], cb[name]), name
            seen = (ca["id"] >= 0).nonzero().squeeze(-1)
            for name in ("k", "v"):
                assert_parity(cb[name][:, seen], ca[name][:, seen].float())


def test_noalloc_rejects_calls_beyond_the_scratch(cuda_device):
    blk = make_oracle_block(256, 512, 2, seed=78)
    nb = NativeBlock(to_device_block(blk))
    B, Q, D = 1, 8192, 256   # ~46 MB of scratch at this shape
    x = torch.zeros(B, Q, D, dtype=torch.bfloat16, device="cuda")
    ctx = torch.zeros(B, 16, D, dtype=torch.bfloat16, device="cuda")
    temb = torch.zeros(B, 1, 6, D, device="cuda")
    out = torch.empty_like(x)
    lib = _lib.load()
    a = nb.make_args(x, ctx, temb, None, None, None, 0, out)
    assert lib.wamb_block_workspace_bytes(a) > _lib.NOALLOC_SCRATCH_BYTES
    assert lib.wamb_block_forward_noalloc(a, _lib.stream_ptr()) == 7  # WAMB_ERR_WORKSPACE
    assert b"no-allocation" in lib.wamb_last_error()
