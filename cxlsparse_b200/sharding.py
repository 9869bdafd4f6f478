"""User sharding across GPUs (one process per GPU), the score gather, and
the KV-head split of a GPU pair.

Per-(user, layer, kv_head) plans are independent (the dedup key includes the
user's cache row), so users are assigned round-robin to ranks and every rank
runs the whole path locally with its own pinned pool slice; the per-user
score outputs are all-gathered after the forward. When the two KV heads of a
user are split over a GPU pair, the attention outputs are exchanged once per
layer through NVLink peer stores (PeerExchange).
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
    """Process groups of the KV-head split (long-history serving, one GPU pair per user set): ranks
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


class _DeviceArray:
    """A device byte range presented through __cuda_array_interface__."""

    def __init__(self, ptr, shape, typestr):
        self.__cuda_array_interface__ = dict(shape=tuple(shape), typestr=typestr,
                                             data=(ptr, False), version=3, strides=None)


class _CudaIpc:
    """Allocation and CUDA IPC through the library (the default for PeerExchange)."""

    def __init__(self, device):
        self.device = device

    def alloc(self, nbytes):
        import ctypes

        from . import _lib
        ptr = ctypes.c_void_p()
        _lib.check(_lib.lib().cxs_device_alloc(nbytes, ctypes.byref(ptr)))
        return ptr.value

    def free(self, ptr):
        from . import _lib
        _lib.check(_lib.lib().cxs_device_free(ptr))

    def handle(self, ptr):
        import ctypes

        from . import _lib
        out = ctypes.create_string_buffer(64)
        _lib.check(_lib.lib().cxs_ipc_get_handle(ptr, out))
        return out.raw

    def open(self, handle):
        import ctypes

        from . import _lib
        ptr = ctypes.c_void_p()
        _lib.check(_lib.lib().cxs_ipc_open_handle(ctypes.create_string_buffer(handle, 64),
                                                  ctypes.byref(ptr)))
        return ptr.value

    def close(self, ptr):
        from . import _lib
        _lib.check(_lib.lib().cxs_ipc_close(ptr))

    def synchronize(self):
        torch.cuda.synchronize(self.device)

    def view(self, ptr, shape, dtype):
        typestr = {torch.bfloat16: "<i2", torch.int32: "<i4"}[dtype]
        t = torch.as_tensor(_DeviceArray(ptr, shape, typestr), device=self.device)
        return t.view(dtype) if dtype == torch.bfloat16 else t


class PeerExchange:
    """Per-layer exchange of a KV-head-split pair over NVLink peer memory.

    Rank `shard` of the pair owns KV heads shard * kv_local ... of every layer.
    Its attention launch stores every output row both into its own gather
    buffer and into its peer's (NVLink stores from the attention epilogue,
    cxs_attend_buffers.out_peer); cxs_exchange_barrier then announces the
    rows and waits, bounded, for the peer's. o_proj reads the local gather
    buffer, which then holds all heads. Two gather buffers alternate by layer
    parity: a rank that runs ahead can reach layer L + 2 only after its peer
    finished layer L + 1's attention, which comes after the peer's layer-L
    o_proj, so no row is overwritten while it is read (layer counts must be
    even for the parity to alternate across forwards). Buffers and flags are
    shared with CUDA IPC; nothing uses NVLink multicast.
    """

    def __init__(self, group, shard, shards, rows, kv_heads, kv_local, device, *,
                 spin_limit=1 << 32, ipc=None):
        import ctypes

        import torch.distributed as dist

        if shards != 2:
            raise ValueError("the peer exchange serves a GPU pair")
        self.shard, self.shards, self.rows = shard, shards, rows
        self.heads, self.head0 = kv_heads, shard * kv_local
        self.spin_limit = spin_limit
        self.ipc = ipc or _CudaIpc(device)
        nbytes = rows * kv_heads * 16 * 64 * 2
        self.local = [self.ipc.alloc(nbytes) for _ in range(2)]
        # control: flags [8] int32 at byte 0, step counter at 64, error word at 128
        self.control = self.ipc.alloc(256)
        mine = [self.ipc.handle(ptr) for ptr in self.local + [self.control]]
        everyone = [None] * shards
        dist.all_gather_object(everyone, mine, group=group)
        self.peer = 1 - shard
        self.remote = [self.ipc.open(h) for h in everyone[self.peer]]
        self.views = [self.ipc.view(ptr, (rows, kv_heads, 16, 64), torch.bfloat16)
                      for ptr in self.local]
        self.error = self.ipc.view(self.control + 128, (1,), torch.int32)
        flags = [0] * shards
        flags[self.peer] = self.remote[2]
        self.peer_flags = (ctypes.c_void_p * shards)(*flags)
        self.group = group

    def targets(self, layer, rows):
        """Where layer `layer`'s attention writes its rows: (local gather buffer,
        peer gather buffer address, heads of the buffer, this rank's first head).
        The launch writes the whole query bucket holding `rows` (padded rows
        included), so the bucket must fit the buffers."""
        from .transport import query_bucket

        if query_bucket(rows) > self.rows:
            raise ValueError(f"{rows} rows (bucket {query_bucket(rows)}) exceed the exchange "
                             f"buffers ({self.rows})")
        b = layer % 2
        return self.views[b], self.remote[b], self.heads, self.head0

    def barrier(self, stream):
        """Enqueue the announce-and-wait step after this layer's attention."""
        from . import _lib
        _lib.check(_lib.lib().cxs_exchange_barrier(
            self.control + 64, self.peer_flags, self.control, self.shard, self.shards,
            self.spin_limit, self.control + 128, stream))

    def check(self):
        """Raise if a barrier wait gave up (reads the device error word)."""
        code = int(self.error.item())
        if code:
            raise RuntimeError(f"KV-head exchange timed out (error word {code:#x})")

    def close(self):
        """Unmap the peer's buffers, then (after the peer has done the same)
        free this rank's."""
        import torch.distributed as dist

        if self.remote is None:
            return
        self.ipc.synchronize()
        for ptr in self.remote:
            self.ipc.close(ptr)
        self.remote = None
        dist.barrier(group=self.group)
        self.views = self.error = None
        for ptr in self.local + [self.control]:
            self.ipc.free(ptr)
