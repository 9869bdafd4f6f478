"""Backing KV pool outside HBM and the hot-replica cache state.

``MemoryPool`` keeps the reference's page allocator and page-striped region
layout (``mempool/pool.py:16-330``, ``mempool/cxl.py:110-113``): a token slot
``s`` lives in page ``s // page_size``; pages are striped round-robin over
``regions``; region ``r`` holds its pages contiguously. On B200 each region is
a NUMA-local anonymous mapping pinned and registered for mapped device access
(device VA == host VA), created by ``cxs_pool_create``; ``backend="dram"``
registers caller-style anonymous memory exactly like the reference's DRAM
pool (``mempool/pool.py:60`` + ``native/cuda_registration.cuh:19-40``).

``HiSparseCache`` holds the residency state the planner reads
(``mempool/hisparse.py:35-139``): ``tags``/``locs`` [rows, hot + 1],
``host_locs`` [rows, max_history] (token -> pool slot) and ``data`` (the HBM
hot replica).
"""

import ctypes

import torch

from . import _lib


class MemoryPool:
    """Token-slot pool of ``dim`` bf16 values per token in pinned host memory."""

    def __init__(self, pages, dim=128, backend="host", *, page_size=64, regions=1,
                 device=None, numa_node=-1):
        if pages <= 0 or dim <= 0 or page_size <= 0 or regions < 1:
            raise ValueError("pages, dim, page_size and regions must be positive")
        if backend not in ("host", "dram"):
            raise ValueError(f"Unknown backend: {backend}")
        self.pages, self.dim, self.backend = pages, dim, backend
        self.page_size, self.regions = page_size, regions
        self.token_bytes = dim * 2
        self.page_bytes = page_size * self.token_bytes
        self.size = pages * self.page_bytes
        self.free = list(range(pages - 1, -1, -1))
        self.allocated = set()
        self.read_bytes = self.write_bytes = 0
        self.read_operations = self.write_operations = 0
        self.read_kernel_launches = self.write_kernel_launches = 0
        self._pending_read_counts = []
        self.device = torch.device("cuda", torch.cuda.current_device() if device is None
                                   else torch.device(device).index or 0)
        self.region_pages = [(pages + regions - 1 - r) // regions for r in range(regions)]
        self._bases, self.numa_nodes = [], []
        self._buffers = []
        lib = _lib.lib()
        for r in range(regions):
            nbytes = max(1, self.region_pages[r]) * self.page_bytes
            if backend == "host":
                base, node = ctypes.c_void_p(), ctypes.c_int32(-1)
                _lib.check(lib.cxs_pool_create(nbytes, self.device.index, numa_node,
                                               ctypes.byref(base), ctypes.byref(node)))
                self._bases.append((base.value, nbytes))
                self.numa_nodes.append(node.value)
            else:
                buffer = torch.zeros(nbytes, dtype=torch.uint8)
                _lib.check(lib.cxs_pool_register(buffer.data_ptr(), nbytes))
                self._buffers.append(buffer)
                self._bases.append((buffer.data_ptr(), nbytes))
                self.numa_nodes.append(-1)
        self.region_bases = torch.tensor([b for b, _ in self._bases], dtype=torch.int64,
                                         device=self.device)
        self.last_use = torch.cuda.Event()
        self.last_use.record(torch.cuda.current_stream(self.device))
        self.closed = False

    # -- reference allocator surface (mempool/pool.py:108-151) --------------
    @property
    def region_count(self):
        return self.regions

    def allocate(self, count):
        if count < 0 or count > len(self.free):
            raise ValueError("Backing pool exhausted")
        slots = [self.free.pop() for _ in range(count)]
        self.allocated.update(slots)
        return slots

    def release(self, slots):
        if len(slots) != len(set(slots)) or any(s not in self.allocated for s in slots):
            raise ValueError("Invalid page release")
        for s in slots:
            self.allocated.remove(s)
            self.free.append(s)

    def token_slot(self, page, offset):
        if page not in self.allocated or not 0 <= offset < self.page_size:
            raise ValueError("Invalid page or token offset")
        return page * self.page_size + offset

    def token_slots(self, pages, start, stop):
        if not 0 <= start <= stop <= len(pages) * self.page_size:
            raise ValueError("Invalid token span")
        slots, cursor = [], start
        while cursor < stop:
            page, offset = divmod(cursor, self.page_size)
            count = min(stop - cursor, self.page_size - offset)
            base = self.token_slot(pages[page], offset)
            slots.extend(range(base, base + count))
            cursor += count
        return slots

    def location(self, slot):
        """(region, local slot) of a global token slot (mempool/cxl.py:110-113)."""
        page, offset = divmod(slot, self.page_size)
        local_page, region = divmod(page, self.regions)
        return region, local_page * self.page_size + offset

    @property
    def pool_tokens(self):
        return self.pages * self.page_size

    # -- IO ------------------------------------------------------------------
    def write_many(self, slots, tensor, *, asynchronous=False):
        """Scatter [n, dim] bf16 records (CUDA) into token slots with one kernel.

        ``slots`` is a sequence or an int64 CUDA tensor of trusted, unique,
        allocated slots (mempool/pool.py:191-233).
        """
        if self.closed:
            raise RuntimeError("pool is closed")
        if tensor.device.type != "cuda" or tensor.dtype != torch.bfloat16:
            raise ValueError("pool writes take bf16 CUDA records")
        tensor = tensor.reshape(-1, self.dim).contiguous()
        if isinstance(slots, torch.Tensor):
            device_slots = slots.to(device=tensor.device, dtype=torch.int64)
        else:
            slots = list(slots)
            device_slots = torch.tensor(slots, dtype=torch.int64, pin_memory=True).to(
                tensor.device, non_blocking=True)
        n = len(device_slots)
        if n != len(tensor):
            raise ValueError("slot count does not match records")
        if not n:
            return
        stream = torch.cuda.current_stream(tensor.device)
        stream.wait_event(self.last_use)
        _lib.check(_lib.lib().cxs_pool_write(
            tensor.data_ptr(), device_slots.data_ptr(), n, self.region_bases.data_ptr(),
            self.regions, self.page_size, stream.cuda_stream))
        self.last_use = torch.cuda.Event()
        self.last_use.record(stream)
        if not asynchronous:
            stream.synchronize()
        self.write_bytes += n * self.token_bytes
        self.write_operations += 1
        self.write_kernel_launches += 1

    def flush_read_stats(self):
        """Resolve deferred per-region read counts once (mempool/pool.py:459-470)."""
        if not self._pending_read_counts:
            return
        pending, self._pending_read_counts = self._pending_read_counts, []
        for counts, launches in pending:
            self.read_bytes += int(counts.sum().item()) * self.token_bytes
            self.read_operations += launches
            self.read_kernel_launches += launches

    def close(self):
        if self.closed:
            return
        torch.cuda.synchronize(self.device)
        lib = _lib.lib()
        for (base, nbytes), buffer in zip(self._bases, self._buffers or [None] * self.regions):
            if self.backend == "host":
                _lib.check(lib.cxs_pool_destroy(base, nbytes))
            else:
                _lib.check(lib.cxs_pool_unregister(base))
        self._buffers = []
        self.closed = True

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class HiSparseCache:
    """Token-granular hot replica plus the token -> pool slot table."""

    def __init__(self, pool, rows=32, max_history=4096, hot=32, topk=8, dim=128):
        if not (0 < topk <= hot <= 16384) or hot & (hot - 1):
            raise ValueError("hot must be a power of two, topk <= hot <= 16384")
        self.pool, self.rows, self.max_history = pool, rows, max_history
        self.hot, self.topk, self.dim = hot, topk, dim
        device = pool.device
        self.tags = torch.full((rows, hot + 1), -1, dtype=torch.int32, device=device)
        self.locs = torch.arange(rows * (hot + 1), dtype=torch.int32,
                                 device=device).reshape(rows, hot + 1)
        self.host_locs = torch.full((rows, max_history), -1, dtype=torch.int64, device=device)
        self.data = torch.zeros((rows * (hot + 1), dim), dtype=torch.bfloat16, device=device)
        self.last_use = torch.cuda.Event()
        self.last_use.record(torch.cuda.current_stream(device))
        self.has_last_use = True
        self.planner_calls = 0
        self.bound_lengths = [0] * rows
        self.replica_locs = None  # optional residency table (enable_replica)
        self.replica = None
        self.replica_used = 0

    def enable_replica(self, capacity):
        """A static HBM replica of up to ``capacity`` history tokens with a
        per-token residency table ``replica_locs[row, token]`` (replica slot
        or -1). Unlike the hot hash (at most ``hot`` tokens per row, refreshed
        by the frequency policy), the table holds any residency pattern of
        any size: the most recent N blocks, interleaved or partly resident
        blocks. Not in the reference, whose replica is the hot hash."""
        device = self.data.device
        self.replica_locs = torch.full((self.rows, self.max_history), -1, dtype=torch.int32,
                                       device=device)
        self.replica = torch.zeros((max(1, capacity), self.dim), dtype=torch.bfloat16,
                                   device=device)
        self.replica_used = 0

    def replicate(self, row, tokens, records):
        """Make history ``tokens`` (device int64 [n]) of ``row`` resident in the
        replica with their KV ``records`` [n, dim]."""
        n = len(tokens)
        if self.replica_locs is None or self.replica_used + n > len(self.replica):
            raise ValueError("replica disabled or full")
        if not n:
            return
        stream = torch.cuda.current_stream(self.data.device)
        stream.wait_event(self.last_use)
        slots = torch.arange(self.replica_used, self.replica_used + n, dtype=torch.int32,
                             device=self.data.device)
        self.replica[slots.long()] = records
        self.replica_locs[row, tokens] = slots
        self.replica_used += n
        self.last_use.record(stream)

    def bind(self, row, slots):
        stream = torch.cuda.current_stream(self.data.device)
        stream.wait_event(self.last_use)
        self.host_locs[row].fill_(-1)
        if len(slots):
            self.host_locs[row, : len(slots)] = torch.as_tensor(
                slots, dtype=torch.int64).to(self.data.device)
        self.last_use.record(stream)
        self.bound_lengths[row] = len(slots)

    def append_slots(self, row, start, slots):
        """Upload an append-only history suffix (mempool/hisparse.py:122-139)."""
        if not 0 <= row < self.rows or start != self.bound_lengths[row] or \
                start + len(slots) > self.max_history:
            raise ValueError("Invalid append-only history binding")
        if not len(slots):
            return
        stream = torch.cuda.current_stream(self.data.device)
        stream.wait_event(self.last_use)
        self.host_locs[row, start:start + len(slots)] = torch.as_tensor(
            slots, dtype=torch.int64).to(self.data.device, non_blocking=True)
        self.last_use.record(stream)
        self.bound_lengths[row] += len(slots)
