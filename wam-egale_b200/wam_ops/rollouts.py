"""Rollout sharding across GPUs (one process per GPU).

Independent rollouts (and speculative draft branches) are the only axis the
denoise step shards on: every rank holds the full weights and its own
contiguous slice of rollouts with their KV pools, runs the step with no
data-path collective, and the per-rollout action outputs are all-gathered
afterwards (NCCL over NVLink on GPUs; gloo works for CPU tests).
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
