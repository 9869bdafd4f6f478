"""Multi-rank host logic on CPU: user sharding and the score all-gather (gloo, 2 ranks)."""

import os
import socket

import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cxlsparse_b200.sharding import PeerExchange, gather_scores, head_pair_groups, users_for_rank


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


class _FakeIpc:
    """Stands in for CUDA IPC on CPU: addresses are (rank, serial) codes."""

    def __init__(self, rank):
        self.rank, self.serial, self.log = rank, 0, []

    def alloc(self, nbytes):
        self.serial += 1
        return (self.rank + 1) * 1_000_000 + self.serial * 1000

    def free(self, ptr):
        self.log.append(("free", ptr))

    def handle(self, ptr):
        return ptr.to_bytes(8, "little") + bytes(56)

    def open(self, handle):
        ptr = int.from_bytes(handle[:8], "little")
        self.log.append(("open", ptr))
        return ptr + 7  # where this process maps the peer's allocation

    def close(self, ptr):
        self.log.append(("close", ptr))

    def synchronize(self):
        pass

    def view(self, ptr, shape, dtype):
        return torch.full(shape, ptr % 1_000_000, dtype=torch.float32).to(dtype)


def _head_worker(rank, world, port, results):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        group, shard, shards, pair, pairs = head_pair_groups(world)
        ipc = _FakeIpc(rank)
        exchange = PeerExchange(group, shard, shards, rows=64, kv_heads=2, kv_local=1,
                                device="cpu", ipc=ipc)
        layers = [exchange.targets(layer, 8) for layer in range(4)]
        try:  # 70 rows are padded to a 128-row bucket: larger than the buffers
            exchange.targets(0, 70)
            oversized = False
        except ValueError:
            oversized = True
        peer_flags = [int(p or 0) for p in exchange.peer_flags]
        remote = list(exchange.remote)
        exchange.close()
        results[rank] = (shard, shards, pair, pairs,
                         [(view.shape, float(view[0, 0, 0, 0]), peer, heads, head0)
                          for view, peer, heads, head0 in layers],
                         peer_flags, remote, ipc.log, oversized)
    finally:
        dist.destroy_process_group()


def test_head_pairs_exchange_buffers():
    """Each rank of a pair maps its peer's two gather buffers and flag block,
    alternates the buffers by layer, writes its own head slot, and unmaps the
    peer's memory before freeing its own."""
    world = 4
    manager = mp.get_context("spawn").Manager()
    results = manager.dict()
    mp.start_processes(_head_worker, args=(world, _free_port(), results), nprocs=world,
                       start_method="spawn")
    for rank in range(world):
        shard, shards, pair, pairs, layers, peer_flags, remote, log, oversized = results[rank]
        assert oversized
        assert (shard, shards, pair, pairs) == (rank % 2, 2, rank // 2, 2)
        peer = rank ^ 1
        peer_allocs = [(peer + 1) * 1_000_000 + k * 1000 for k in (1, 2, 3)]
        assert remote == [a + 7 for a in peer_allocs]
        assert peer_flags[shard] == 0 and peer_flags[1 - shard] == peer_allocs[2] + 7
        for layer, (shape, local_code, peer_ptr, heads, head0) in enumerate(layers):
            assert tuple(shape) == (64, 2, 16, 64) and heads == 2 and head0 == shard
            assert local_code == (1 + layer % 2) * 1000        # own buffer of this parity
            assert peer_ptr == peer_allocs[layer % 2] + 7     # peer's buffer, same parity
        closes = [i for i, (op, _) in enumerate(log) if op == "close"]
        frees = [i for i, (op, _) in enumerate(log) if op == "free"]
        assert len(closes) == 3 and len(frees) == 3 and max(closes) < min(frees)
