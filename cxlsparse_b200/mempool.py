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
from array import array

import torch

from . import _lib


class PageAllocator:
    """Ownership of the pool's pages.

    Free pages sit on a stack. A fresh pool hands pages out in ascending order
    (0, 1, 2, ...); released pages come back on top, so the most recently
    released page is handed out first. That is the order of the reference
    allocator (``mempool/pool.py:100-125``), and the slot numbers of the
    planner fixtures depend on it. Ownership is one flag per page, so checks
    cost O(1) per page.
    """

    def __init__(self, pages):
        self._owned = bytearray(pages)
        self._stack = array("q", range(pages - 1, -1, -1))  # top of stack = last item

    @property
    def free_pages(self):
        return len(self._stack)

    def owns(self, page):
        return 0 <= page < len(self._owned) and self._owned[page] == 1

    def allocate(self, count):
        if not 0 <= count <= len(self._stack):
            raise ValueError("Backing pool exhausted")
        keep = len(self._stack) - count
        taken = self._stack[keep:].tolist()[::-1]
        del self._stack[keep:]
        for page in taken:
            self._owned[page] = 1
        return taken

    def release(self, pages):
        pages = list(pages)
        if len(set(pages)) != len(pages) or not all(self.owns(p) for p in pages):
            raise ValueError("Invalid page release")
        for page in pages:
            self._owned[page] = 0
        self._stack.extend(pages)


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
        self.pages_owned = PageAllocator(pages)
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
        return self.pages_owned.allocate(count)

    def release(self, slots):
        self.pages_owned.release(slots)

    def token_slot(self, page, offset):
        if not self.pages_owned.owns(page) or not 0 <= offset < self.page_size:
            raise ValueError("Invalid page or token offset")
        return page * self.page_size + offset

    def token_slots(self, pages, start, stop):
        """Slots of token positions [start, stop) of a history laid out over
        ``pages`` (position t lives at offset t % page_size of pages[t //
        page_size]); each page is validated once."""
        size = self.page_size
        if not 0 <= start <= stop <= len(pages) * size:
            raise ValueError("Invalid token span")
        slots = []
        for index in range(start // size, -(-stop // size)):
            lo, hi = max(start, index * size), min(stop, (index + 1) * size)
            shift = self.token_slot(pages[index], 0) - index * size
            slots.extend(range(lo + shift, hi + shift))
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

    def _store_slots(self, row, start, slots, *, clear):
        """Write pool slots of tokens [start, start + len(slots)) of ``row``
        into the token -> slot table, ordered after earlier users of the
        table (``last_use``)."""
        stream = torch.cuda.current_stream(self.data.device)
        stream.wait_event(self.last_use)
        table = self.host_locs[row]
        if clear:
            table.fill_(-1)
        if len(slots):
            table[start:start + len(slots)].copy_(torch.as_tensor(slots, dtype=torch.int64))
        self.last_use.record(stream)

    def bind(self, row, slots):
        """Replace the whole history binding of ``row``."""
        self._store_slots(row, 0, slots, clear=True)
        self.bound_lengths[row] = len(slots)

    def append_slots(self, row, start, slots):
        """Extend the binding of ``row`` by a suffix that starts where the
        bound history ends; earlier slots stay as they are
        (``mempool/hisparse.py:122-139``)."""
        if (not 0 <= row < self.rows or start != self.bound_lengths[row]
                or start + len(slots) > self.max_history):
            raise ValueError("Invalid append-only history binding")
        if len(slots):
            self._store_slots(row, start, slots, clear=False)
            self.bound_lengths[row] += len(slots)
