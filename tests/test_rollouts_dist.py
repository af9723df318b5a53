"""Rollout sharding, the action-output gather and the KV-history broadcast
of split candidate verification on 2 CPU ranks (gloo): the host-side logic
of the multi-GPU bench paths, without a GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import wan_block as ob
from wam_ops.rollouts import broadcast_cache, gather_actions, shard


def test_shard_covers_all_rollouts():
    for total in (0, 1, 7, 8, 64, 65):
        for world in (1, 2, 3, 8):
            parts = [shard(total, world, r) for r in range(world)]
            assert [i for p in parts for i in p] == list(range(total))
            assert max(map(len, parts)) - min(map(len, parts)) <= 1
    with pytest.raises(ValueError):
        shard(8, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    port = s.getsockname()[1]
    s.close()
    return port


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        total, Q, D, A = 8, 12, 16, 4
        mine = shard(total, world, rank)
        # rollout r's hidden state is filled with r (stand-in for a step output)
        hidden = torch.stack([torch.full((Q, D), float(r)) for r in mine])
        out = gather_actions(hidden, A)
        expect = torch.stack([torch.full((A, D), float(r)) for r in range(total)])
        q.put((rank, bool(torch.equal(out, expect))))
    finally:
        dist.destroy_process_group()


def test_gather_actions_two_ranks():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    results = dict(q.get(timeout=5) for _ in procs)
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: True, 1: True}


def test_gather_without_group_is_local():
    h = torch.arange(2 * 5 * 3.0).view(2, 5, 3)
    assert torch.equal(gather_actions(h, 2), h[:, -2:])


def _verify_worker(rank, world, port, q):
    """Candidates split across ranks over a history that only rank 0
    filled: after broadcast_cache every rank's cache equals rank 0's, and
    the gathered candidate outputs equal one rank verifying all of them."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        torch.manual_seed(0)
        D, H, F, pool, hist, Q, ncand = 128, 1, 256, 48, 32, 8, 4
        blk = ob.WanTransformerBlock(D, F, H, cross_attn_norm=True).eval()
        for prm in blk.parameters():    # same weights on every rank (same seed)
            torch.nn.init.normal_(prm, std=0.05)
        blk.attn1.init_kv_cache("pos", pool, H, 128, "cpu", torch.float32, 1)
        c = blk.attn1.attn_caches["pos"]
        c["k"].zero_(), c["v"].zero_()
        if rank == 0:                   # only rank 0 holds the history
            g = torch.Generator().manual_seed(1)
            c["k"].copy_(torch.randn(c["k"].shape, generator=g))
            c["v"].copy_(torch.randn(c["v"].shape, generator=g))
            c["mask"][:hist] = True
            c["id"][:hist] = torch.arange(hist) // 16
        nbytes = broadcast_cache([blk])
        g = torch.Generator().manual_seed(2)
        x = torch.randn(ncand, Q, D, generator=g)
        ctx = torch.randn(1, 8, D, generator=g).expand(ncand, -1, -1)
        temb = torch.randn(ncand, Q, 6, D, generator=g) * 0.1
        rows = torch.zeros(ncand, dtype=torch.long)
        with torch.no_grad():
            full = blk(x, ctx, temb, None, candidate_cache_rows=rows)
            mine = list(shard(ncand, world, rank))
            part = blk(x[mine], ctx[mine], temb[mine], None, candidate_cache_rows=rows[mine])
        gathered = gather_actions(part, Q)
        q.put((rank, nbytes == sum(t.numel() * t.element_size() for t in c.values()),
               bool(torch.allclose(gathered, full, atol=1e-5)), int(c["mask"].sum())))
    finally:
        dist.destroy_process_group()


def test_split_candidates_with_broadcast_history():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_verify_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
    results = dict((r[0], r[1:]) for r in (q.get(timeout=5) for _ in procs))
    assert all(p.exitcode == 0 for p in procs)
    assert results == {0: (True, True, 32), 1: (True, True, 32)}
