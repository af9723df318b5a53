"""Rollout sharding and the action-output gather on 2 CPU ranks (gloo):
the host-side logic of the multi-GPU bench path, without a GPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from wam_ops.rollouts import gather_actions, shard


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
