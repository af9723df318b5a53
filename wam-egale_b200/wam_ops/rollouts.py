"""Rollout and draft-branch sharding across GPUs (one process per GPU).

Independent rollouts (and speculative draft branches) are the only axis the
denoise step shards on: every rank holds the full weights and its own
contiguous slice of rollouts with their KV pools, runs the step with no
data-path collective, and the per-rollout action outputs are all-gathered
afterwards (NCCL over NVLink on GPUs; gloo works for CPU tests).

Candidate verification on several GPUs (a speculative verify batch split
across ranks, the candidate path of model.py:624-660 and
wan_va_server.py:1906-1930) needs the candidates' shared, read-only KV
history on every rank: broadcast_cache copies each layer's cache from one
rank into the others' own memory once, and shard() gives each rank its
candidates.
"""
import torch
import torch.distributed as dist


def shard(total, world, rank):
    """Contiguous rollout indices of `rank`: sizes differ by at most one."""
    if not (0 <= rank < world) or total < 0:
        raise ValueError("bad shard request")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def gather_actions(hidden, action_tokens, group=None):
    """All-gather the last `action_tokens` rows of every local rollout:
    hidden [b, Q, D] -> [world * b, action_tokens, D] in rank order (equal b
    on every rank). Without an initialised process group it returns the
    local slice."""
    local = hidden[:, -action_tokens:].contiguous()
    if not (dist.is_available() and dist.is_initialized()):
        return local
    world = dist.get_world_size(group)
    out = torch.empty((world * local.shape[0],) + tuple(local.shape[1:]), dtype=local.dtype,
                      device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local, group=group)
    else:
        dist.all_gather(list(out.chunk(world)), local, group=group)
    return out


def broadcast_cache(blocks, src=0, cache_name="pos", group=None):
    """Broadcast every layer's self-attention cache (k, v, id, mask,
    is_pred) from rank `src` into the same tensors on the other ranks, once
    (each rank then reads its own copy; nothing crosses the links during a
    step). The caches must exist on every rank with equal shapes. Returns
    the bytes received per rank."""
    nbytes = 0
    for blk in blocks:
        cache = blk.attn1.attn_caches[cache_name]
        for name in ("k", "v", "id", "mask", "is_pred"):
            t = cache[name]
            if t.dtype == torch.bool:
                # gloo has no bool reduction type; the bytes are the same
                view = t.view(torch.uint8)
                dist.broadcast(view, src, group=group)
            else:
                dist.broadcast(t, src, group=group)
            nbytes += t.numel() * t.element_size()
    return nbytes
