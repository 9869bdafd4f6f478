"""Multi-rank host logic on CPU: user sharding and the score all-gather (gloo, 2 ranks)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cxlsparse_b200.sharding import (gather_scores, head_exchange, head_pair_groups,
                                     users_for_rank)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        users = users_for_rank(list(range(7)), rank, world)
        local = torch.tensor([float(sum(users)), float(len(users))])
        gathered = gather_scores(local)
        results[rank] = (users, gathered.tolist())
    finally:
        dist.destroy_process_group()


def test_round_robin_users_and_gather():
    world = 2
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_worker, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn")
    assert results[0][0] == [0, 2, 4, 6] and results[1][0] == [1, 3, 5]
    expected = [[12.0, 4.0], [9.0, 3.0]]
    assert results[0][1] == expected and results[1][1] == expected


def test_assignment_covers_every_user_once():
    users = list(range(64))
    for world in (1, 2, 4, 8):
        seen = sorted(u for r in range(world) for u in users_for_rank(users, r, world))
        assert seen == users


def _head_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        group, shard, shards, pair, pairs = head_pair_groups(world)
        exchange = head_exchange(group, shards)
        # [E=3, kv_local=1, 16, 64]: head value = 100 * (global head) + token
        local = torch.zeros(3, 1, 16, 64)
        for e in range(3):
            local[e] = 100 * (shard + 0) + e + 1000 * pair
        full = exchange(local)
        results[rank] = (shard, shards, pair, pairs, full[:, :, 0, 0].tolist())
    finally:
        dist.destroy_process_group()


def test_head_pairs_exchange_attention_outputs():
    world = 4
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_head_worker, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn")
    for rank in range(world):
        shard, shards, pair, pairs, heads = results[rank]
        assert (shard, shards, pair, pairs) == (rank % 2, 2, rank // 2, 2)
        # token e: [head 0 of the pair, head 1 of the pair]
        assert heads == [[1000 * pair + e, 1000 * pair + 100 + e] for e in range(3)]
