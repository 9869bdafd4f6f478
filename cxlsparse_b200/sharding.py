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


def head_pair_groups(world):
    """Process groups of the KV-head split: ranks
    (0, 1), (2, 3), ... each serve one set of users, rank 2p + i owning KV
    head i of every layer. Every rank must call this (new_group is collective);
    returns (group of this rank, shard index, shard count, pair index, pairs)."""
    import torch.distributed as dist

    if world == 1:
        return None, 0, 1, 0, 1
    if world % 2:
        raise ValueError("the KV-head split needs an even number of ranks")
    rank = dist.get_rank()
    mine = None
    for pair in range(world // 2):
        group = dist.new_group([2 * pair, 2 * pair + 1])
        if rank // 2 == pair:
            mine = group
    return mine, rank % 2, 2, rank // 2, world // 2


def head_exchange(group, shards):
    """Per-layer exchange of a head-sharded model: every rank of `group` holds
    the attention output of its own KV heads [E, kv_local, 16, 64]; the
    all-gather returns all heads' [E, kv_local * shards, 16, 64] in head order
    (rank r of the group owns heads r * kv_local ...)."""
    import torch.distributed as dist

    def exchange(local):
        local = local.contiguous()
        gathered = torch.empty((shards,) + tuple(local.shape), dtype=local.dtype,
                               device=local.device)
        dist.all_gather_into_tensor(gathered.view(-1), local.view(-1), group=group)
        return gathered.transpose(0, 1).reshape(local.shape[0], shards * local.shape[1],
                                                *local.shape[2:])

    return exchange
