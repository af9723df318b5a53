"""tcgen05 flash attention (wamb_attention) against torch SDPA in fp32.

Tolerance: P is rounded to bf16 before the PV product and the output once to
bf16, so |out - ref| <= 1e-2 + 2e-2 * |ref| on N(0,1) inputs.
"""
import pytest
import torch
import torch.nn.functional as F

from wam_ops import _lib, ops

pytestmark = pytest.mark.gpu


def _sdpa_ref(q, k, v):
    """q [B,Sq,H,d], k/v [B,Sk,H,d] -> fp32 [B,Sq,H,d]."""
    o = F.scaled_dot_product_attention(q.float().transpose(1, 2), k.float().transpose(1, 2),
                                       v.float().transpose(1, 2))
    return o.transpose(1, 2)


def _check(out, ref):
    out = out.float()
    assert torch.isfinite(out).all()
    err = (out - ref).abs()
    bound = 1e-2 + 2e-2 * ref.abs()
    assert (err <= bound).all(), f"max err {err.max().item()}"
    cos = F.cosine_similarity(out.flatten(), ref.flatten(), dim=0).item()
    assert cos >= 0.9999, cos


@pytest.mark.parametrize("B,H,Sq,Sk", [(1, 1, 128, 128), (2, 3, 40, 24), (1, 2, 300, 700),
                                       (2, 2, 7, 1), (1, 4, 129, 257), (3, 1, 1, 513)])
def test_sdpa_contiguous(cuda_device, B, H, Sq, Sk):
    g = torch.Generator(device="cuda").manual_seed(B * 1000 + Sq * 7 + Sk)
    q = torch.randn(B, Sq, H, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Sk, H, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Sk, H, 128, device="cuda", generator=g).bfloat16()
    _check(ops.sdpa(q, k, v), _sdpa_ref(q, k, v))


def _tiles(mask):
    """Host restatement of the kernel's tile list: maximal runs of visible
    slots inside each 128-slot window."""
    m = mask.cpu().tolist()
    out = []
    for i, on in enumerate(m):
        if on and (i % 128 == 0 or not m[i - 1]):
            e = i + 1
            while e < len(m) and e % 128 != 0 and m[e]:
                e += 1
            out.append((i, e - i))
    return out


@pytest.mark.parametrize("pool,density", [(700, 1.0), (700, 0.6), (300, 0.1), (1000, 0.97)])
def test_pool_tiles_ignore_stale_slots(cuda_device, pool, density):
    """Keys read in place from a pool through a tile list; unused slots hold
    NaN and must not leak into the output."""
    g = torch.Generator(device="cuda").manual_seed(pool)
    B, H, Q = 2, 2, 50
    kp = torch.randn(B, pool, H, 128, device="cuda", generator=g).bfloat16()
    vp = torch.randn(B, pool, H, 128, device="cuda", generator=g).bfloat16()
    mask = torch.rand(pool, device="cuda", generator=g) < density
    mask[3] = True
    kp[:, ~mask] = float("nan")
    vp[:, ~mask] = float("nan")
    q = torch.randn(B, Q, H, 128, device="cuda", generator=g).bfloat16()
    tl = _tiles(mask)
    tiles = torch.tensor(tl, dtype=torch.int32, device="cuda").view(-1, 2)
    n = torch.tensor([len(tl)], dtype=torch.int32, device="cuda")
    out = ops.attention(q.view(B * Q, -1), kp.view(B * pool, -1), vp.view(B * pool, -1), heads=H,
                        q_rows=Q, src0_batch_stride=pool, tiles=tiles, n_tiles=n)
    idx = mask.nonzero().squeeze(-1)
    ref = _sdpa_ref(q, kp[:, idx], vp[:, idx])
    _check(out.view(B, Q, H, 128), ref)


def test_candidate_two_sources(cuda_device):
    """History rows selected by a row map plus each candidate's own K/V
    (model.py:654-660)."""
    g = torch.Generator(device="cuda").manual_seed(5)
    Bp, pool, B, H, Q = 2, 400, 4, 2, 32
    kp = torch.randn(Bp, pool, H, 128, device="cuda", generator=g).bfloat16()
    vp = torch.randn(Bp, pool, H, 128, device="cuda", generator=g).bfloat16()
    mask = torch.zeros(pool, dtype=torch.bool, device="cuda")
    mask[:250] = True
    mask[300:350] = True
    rows = torch.tensor([0, 1, 0, 0], dtype=torch.int64, device="cuda")
    qkv = torch.randn(B * Q, 3 * H * 128, device="cuda", generator=g).bfloat16()
    tl = _tiles(mask)
    tiles = torch.tensor(tl, dtype=torch.int32, device="cuda").view(-1, 2)
    n = torch.tensor([len(tl)], dtype=torch.int32, device="cuda")
    D = H * 128
    out = ops.attention(qkv, kp.view(Bp * pool, -1), vp.view(Bp * pool, -1), heads=H, q_rows=Q,
                        src0_batch_stride=pool, tiles=tiles, n_tiles=n, src0_map=rows,
                        k1=qkv, v1=qkv, k1_col=D, v1_col=2 * D)
    idx = mask.nonzero().squeeze(-1)
    q = qkv[:, :D].view(B, Q, H, 128)
    k_own = qkv[:, D:2 * D].view(B, Q, H, 128)
    v_own = qkv[:, 2 * D:].view(B, Q, H, 128)
    k = torch.cat([kp[:, idx].index_select(0, rows), k_own], 1)
    v = torch.cat([vp[:, idx].index_select(0, rows), v_own], 1)
    _check(out.view(B, Q, H, 128), _sdpa_ref(q, k, v))


def test_broadcast_source(cuda_device):
    g = torch.Generator(device="cuda").manual_seed(6)
    B, H, Q, C = 3, 2, 70, 200
    q = torch.randn(B * Q, H * 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(C, H * 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(C, H * 128, device="cuda", generator=g).bfloat16()
    out = ops.attention(q, k, v, heads=H, q_rows=Q, src0_batch_stride=C, src0_len=C, src0_broadcast=True)
    ref = _sdpa_ref(q.view(B, Q, H, 128), k.view(1, C, H, 128).expand(B, -1, -1, -1),
                    v.view(1, C, H, 128).expand(B, -1, -1, -1))
    _check(out.view(B, Q, H, 128), ref)


@pytest.mark.parametrize("Sq,Sk,hot", [(100, 1000, "first"), (100, 1000, "second"), (128, 3553, "last"),
                                       (77, 257, "none"), (384, 1900, "second")])
def test_split_kv_single_tile(cuda_device, Sq, Sk, hot):
    """A CTA holding one query tile runs the first half of the key tiles on
    TMEM slot A and the second half on slot B, then merges the two partial
    softmaxes. Keys scaled up in one half put the row max (and the 2^8 rescale
    steps) in that half only, so a wrong merge weight shows."""
    g = torch.Generator(device="cuda").manual_seed(Sq * 31 + Sk)
    B, H = 2, 2
    q = torch.randn(B, Sq, H, 128, device="cuda", generator=g)
    k = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    v = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    if hot == "first":
        k[:, : Sk // 4] *= 3
    elif hot == "second":
        k[:, -Sk // 4:] *= 3
    elif hot == "last":
        k[:, -5:] *= 4
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    _check(ops.sdpa(q, k, v), _sdpa_ref(q, k, v))


@pytest.mark.parametrize("Sq,Sk,hot", [(300, 1000, "second"), (300, 1000, "last"), (256, 2000, "first"),
                                       (880, 700, "ramp"), (200, 130, "second")])
def test_transposed_output_rescale(cuda_device, Sq, Sk, hot):
    """Queries longer than one tile at one wave run attn_ot_kernel (O^T in
    TMEM, P V as N 256 MMAs). Keys scaled up late make row maxima grow past
    the 2^8 threshold after O^T holds earlier tiles, so the rescale of O^T
    columns by all softmax warps is exercised; "ramp" grows every tile."""
    g = torch.Generator(device="cuda").manual_seed(Sq * 7 + Sk)
    B, H = 1, 2
    q = torch.randn(B, Sq, H, 128, device="cuda", generator=g)
    k = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    v = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    if hot == "first":
        k[:, : Sk // 4] *= 3
    elif hot == "second":
        k[:, Sk // 2:] *= 3
    elif hot == "last":
        k[:, -7:] *= 5
    else:
        k *= torch.linspace(0.5, 4.0, Sk, device="cuda")[None, :, None, None]
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    out = ops.sdpa(q, k, v)
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    _check(out, _sdpa_ref(q, k, v))


@pytest.mark.parametrize("Q,rows,pool,vis", [
    (32, [0, 0, 0, 0], 700, 600),              # G 4: one cluster, one shared history row
    (32, [1, 1, 1, 1, 0, 0, 0, 0], 700, 650),  # two clusters, each with its own history row
    (64, [1, 1], 1000, 930),                   # G 2
    (16, [0] * 8, 500, 420),                   # G 8
    (32, [0, 0, 0, 0], 200, 60),               # two key tiles for four CTAs: some take none
    (32, [0, 0], 700, 600),                    # G 2, R 4: each CTA merges 8 rows of a candidate
    (32, [0], 700, 600),                       # one candidate, 8 CTAs of 4 rows each
    (32, [0, 0, 0], 1000, 900),                # G 3, R 2: a 6-CTA cluster
    (32, [0, 1], 700, 600),                    # rows differ: each candidate alone, R - 1 CTAs idle
    (128, [1], 1000, 1000),                    # a 128-row candidate split over 8 CTAs
])
def test_candidate_grouped(cuda_device, Q, rows, pool, vis):
    """Candidates that share one history row attend as one query group per
    head: a cluster of G candidates (G * Q <= 128) and R CTAs per candidate
    splits the history tiles and the block-diagonal tile of the candidates'
    own keys, then merges (m, l, O) across the cluster. Each candidate must
    still see only the history plus its own keys (model.py:654-660)."""
    g = torch.Generator(device="cuda").manual_seed(Q * 100 + pool)
    Bp, B, H = 2, len(rows), 2
    kp = torch.randn(Bp, pool, H, 128, device="cuda", generator=g).bfloat16()
    vp = torch.randn(Bp, pool, H, 128, device="cuda", generator=g).bfloat16()
    mask = torch.zeros(pool, dtype=torch.bool, device="cuda")
    mask[torch.randperm(pool, generator=g, device="cuda")[:vis]] = True
    kp[:, ~mask] = float("nan")
    vp[:, ~mask] = float("nan")
    r = torch.tensor(rows, dtype=torch.int64, device="cuda")
    D = H * 128
    qkv = torch.randn(B * Q, 3 * D, device="cuda", generator=g).bfloat16()
    tl = _tiles(mask)
    tiles = torch.tensor(tl, dtype=torch.int32, device="cuda").view(-1, 2)
    n = torch.tensor([len(tl)], dtype=torch.int32, device="cuda")
    out = ops.attention(qkv, kp.view(Bp * pool, -1), vp.view(Bp * pool, -1), heads=H, q_rows=Q,
                        src0_batch_stride=pool, tiles=tiles, n_tiles=n, src0_map=r,
                        k1=qkv, v1=qkv, k1_col=D, v1_col=2 * D)
    idx = mask.nonzero().squeeze(-1)
    q = qkv[:, :D].view(B, Q, H, 128)
    k = torch.cat([kp[:, idx].index_select(0, r), qkv[:, D:2 * D].view(B, Q, H, 128)], 1)
    v = torch.cat([vp[:, idx].index_select(0, r), qkv[:, 2 * D:].view(B, Q, H, 128)], 1)
    torch.cuda.synchronize()
    from wam_ops import _lib
    assert _lib.device_status() == 0
    _check(out.view(B, Q, H, 128), _sdpa_ref(q, k, v))


@pytest.mark.parametrize("B,H,Sq,Sk,splits", [
    (1, 24, 880, 4400, 0),     # one cfg2 chunk: one wave of items, the O^T kernel unsplit
    (8, 4, 880, 700, 0),       # 128 items: the O^T kernel, partial last key tile
    (1, 24, 880, 4400, 3),     # forced 3 splits: the split-key kernel
    (1, 3, 300, 1000, 2),      # two-tile items and a single-tile item
    (2, 2, 100, 700, 4),       # single-tile items only, 4 splits
    (1, 2, 256, 512, 3),       # splits of one or two key tiles
])
def test_split_keys(cuda_device, B, H, Sq, Sk, splits):
    """Split-key attention (the CTAs of one (query tile pair, head) item
    take consecutive key ranges and the last of them merges the partials)
    against torch SDPA, bitwise repeatable, with the counters left zero."""
    g = torch.Generator(device="cuda").manual_seed(Sq * 31 + Sk + splits)
    q = torch.randn(B, Sq, H, 128, device="cuda", generator=g).bfloat16()
    k = torch.randn(B, Sk, H, 128, device="cuda", generator=g).bfloat16()
    v = torch.randn(B, Sk, H, 128, device="cuda", generator=g).bfloat16()
    args = dict(heads=H, q_rows=Sq, src0_batch_stride=Sk, src0_len=Sk, kv_splits=splits)
    run = lambda: ops.attention(q.view(B * Sq, H * 128), k.view(B * Sk, H * 128),  # noqa: E731
                                v.view(B * Sk, H * 128), **args)
    out, again = run(), run()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    _check(out.view(B, Sq, H, 128), _sdpa_ref(q, k, v))
    assert torch.equal(out, again)
    ws = ops._SPLIT.get(torch.cuda.current_device())
    if ws is not None:
        assert bool((ws[:8192] == 0).all())


def _split_counters_zero():
    ws = ops._SPLIT.get(torch.cuda.current_device())
    return ws is None or bool((ws[:8192] == 0).all())


@pytest.mark.parametrize("B,H,Sq,Sk,hot", [
    (1, 24, 880, 4400, None),      # one cfg2 chunk: 96 items over 148 CTAs, items over 2-3 CTAs
    (1, 24, 880, 4400, "ramp"),    # maxima grow in every tile: partials with different m
    (1, 24, 520, 3000, "second"),  # 72 items, up to 4 CTAs per item, last pair tile A only
    (3, 16, 600, 1900, None),      # 144 items, every third pair tile A only
    (1, 40, 300, 5000, "last"),    # hot keys in the last segment of each item
    (3, 24, 880, 2000, None),      # 288 items (1.95 waves), all shared by key tiles
    (8, 24, 880, 1100, "second"),  # 768 items: 4 whole waves round-robin, then 176 items shared
    (2, 40, 1592, 1000, None),     # 560 items: 2 whole waves, every seventh pair tile A only
])
def test_stream_k(cuda_device, B, H, Sq, Sk, hot):
    """attn_ot_sk_kernel: whole waves of (query tile pair, head) items
    round-robin, the key tiles of the rest shared over all SMs, partial
    segments merged by the last CTA to finish; bitwise repeatable, counters
    left zero."""
    g = torch.Generator(device="cuda").manual_seed(Sq * 13 + Sk + H)
    q = torch.randn(B, Sq, H, 128, device="cuda", generator=g)
    k = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    v = torch.randn(B, Sk, H, 128, device="cuda", generator=g)
    if hot == "second":
        k[:, Sk // 2:] *= 3
    elif hot == "last":
        k[:, -7:] *= 5
    elif hot == "ramp":
        k *= torch.linspace(0.5, 4.0, Sk, device="cuda")[None, :, None, None]
    q, k, v = q.bfloat16(), k.bfloat16(), v.bfloat16()
    args = dict(heads=H, q_rows=Sq, src0_batch_stride=Sk, src0_len=Sk, kv_splits=0)
    run = lambda: ops.attention(q.view(B * Sq, H * 128), k.view(B * Sk, H * 128),  # noqa: E731
                                v.view(B * Sk, H * 128), **args)
    out, again = run(), run()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    _check(out.view(B, Sq, H, 128), _sdpa_ref(q, k, v))
    assert torch.equal(out, again)
    assert _split_counters_zero()


@pytest.mark.parametrize("visible", ["most", "first300"])
def test_stream_k_pool_and_own_keys(cuda_device, visible):
    """Stream-K over a pool tile list (stale slots hold NaN) followed by the
    call's own K/V as a second source. "first300": the host plans stream-K
    from the pool size, the device finds 3 pool tiles and runs whole items."""
    g = torch.Generator(device="cuda").manual_seed(4400 + len(visible))
    B, H, Q, pool = 1, 24, 880, 4400
    kp = torch.randn(B, pool, H, 128, device="cuda", generator=g).bfloat16()
    vp = torch.randn(B, pool, H, 128, device="cuda", generator=g).bfloat16()
    if visible == "most":
        mask = torch.rand(pool, device="cuda", generator=g) < 0.8
    else:
        mask = torch.zeros(pool, dtype=torch.bool, device="cuda")
        mask[:300] = True
    kp[:, ~mask] = float("nan")
    vp[:, ~mask] = float("nan")
    q = torch.randn(B, Q, H, 128, device="cuda", generator=g).bfloat16()
    k1 = torch.randn(B, Q, H, 128, device="cuda", generator=g).bfloat16()
    v1 = torch.randn(B, Q, H, 128, device="cuda", generator=g).bfloat16()
    tl = _tiles(mask)
    tiles = torch.tensor(tl, dtype=torch.int32, device="cuda").view(-1, 2)
    n = torch.tensor([len(tl)], dtype=torch.int32, device="cuda")
    run = lambda: ops.attention(q.view(B * Q, -1), kp.view(B * pool, -1), vp.view(B * pool, -1),  # noqa: E731
                                heads=H, q_rows=Q, src0_batch_stride=pool, tiles=tiles, n_tiles=n,
                                k1=k1.view(B * Q, -1), v1=v1.view(B * Q, -1), kv_splits=0)
    out, again = run(), run()
    torch.cuda.synchronize()
    assert _lib.device_status() == 0
    idx = mask.nonzero().squeeze(-1)
    ref = _sdpa_ref(q, torch.cat([kp[:, idx], k1], 1), torch.cat([vp[:, idx], v1], 1))
    _check(out.view(B, Q, H, 128), ref)
    assert torch.equal(out, again)
    assert _split_counters_zero()
