"""User sharding across GPUs (one process per GPU) and the score gather.

Per-(user, layer, kv_head) plans are independent (the dedup key includes the
user's cache row), so users are assigned round-robin to ranks and every rank
runs the whole path locally with its own pinned pool slice. The only
collective is the all-gather of per-user score outputs after the forward.
"""

import torch


def users_for_rank(users, rank, world):
    """Round-robin assignment: user u is served by rank u % world."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError("invalid rank / world size")
    return [u for i, u in enumerate(users) if i % world == rank]


def gather_scores(local, group=None):
    """All-gather equally shaped per-rank score tensors -> [world, *local.shape]."""
    import torch.distributed as dist

    world = dist.get_world_size(group)
    flat = torch.empty(world * local.numel(), dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(flat, local.contiguous().view(-1), group=group)
    return flat.view(world, *local.shape)
