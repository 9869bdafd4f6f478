"""GR selected-block transport: the drop-in for the reference's TMA transport.

Mirrors ``cxl_recsys/models/nsa/transport.py:127-706`` (``GRSelectedTransport``
with ``consumer_backend="tma"``): ``run(query, blocks, positions, fetches,
block_size)`` returns ``(output [Q, H, G, 64] bf16, DeferredLayerCounters)``;
the output is a borrowed view valid until the next call (transport.py:703).
Workspaces are cached by shape key with an LRU bound and a byte budget
(transport.py:243-409); plan + fetch/attend can be replayed from a CUDA graph
(transport.py:624-631); the hot-set commit runs once, outside the graph
(transport.py:641).

Besides the reference behaviour, ``run`` accepts the NSA window / compressed
branches and gates (``window=``, ``compressed=``, ``gates=``); the same launch
then returns the gate-mixed attention output of all three branches
(models/nsa/model.py:466-473), so the model needs no separate window or mix
kernels.

All device work goes through ``libcxlsparse_b200.so``; there is no fallback.
"""

import math
import time
from collections import OrderedDict
from dataclasses import dataclass

import torch

from . import _lib
from .planning import ActivePlanAdapter, QueryPrivatePlanAdapter

QUERY_BUCKETS = (64, 128, 256, 512, 1024, 2048, 4096)


class GRWorkspaceLimit(RuntimeError):
    """Capacity refusal before any plan/IO/hot state has been submitted."""


def query_bucket(active_q, buckets=QUERY_BUCKETS):
    """Smallest bucket holding ``active_q`` rows (models/nsa/dispatch.py:25-33)."""
    if active_q < 1:
        raise ValueError("A query bucket requires at least one active row")
    for capacity in buckets:
        if active_q <= capacity:
            return capacity
    raise GRWorkspaceLimit(f"Query length {active_q} exceeds bucket limit {buckets[-1]}")


@dataclass
class DeferredLayerCounters:
    """[H, 7] planner statistics resolved at the forward boundary.

    Columns: unique, unique_old, hits, misses, old_refs, local_refs, errors
    (mempool/device_plan.py:16-42). ``errors`` additionally carries the
    fetch/attend device error word.
    """

    statistics: torch.Tensor
    launches: int
    backend: str = "host"
    device_error: torch.Tensor | None = None

    def materialize(self, rows=None):
        if rows is None:
            rows = self.statistics.tolist()
        if any(row[6] for row in rows):
            raise ValueError(
                "Top-K must contain causal positions or -1 padding, with bound history slots")
        if self.device_error is not None:
            code = int(self.device_error.item())
            if code:
                raise RuntimeError(f"NSA fetch/attend device error word {code:#x}")
        owner = next((i for i, row in enumerate(rows) if row[3]), None)
        return [
            dict(hits=r[2], misses=r[3], old_references=r[4],
                 deduplicated_references=r[4] - r[1], local_tokens=r[5],
                 planner_calls=int(i == 0),
                 h2d_transfers=int(i == owner),
                 fetch_kernel_launches=self.launches if i == 0 else 0)
            for i, r in enumerate(rows)
        ]


def workspace_estimate(queries, cached, heads, groups, width, bs, *, cross_query_dedup=True):
    """Host-known conservative bound (transport.py:90-124)."""
    q = query_bucket(queries)
    logical = max(64, math.ceil((cached + q) / (64 * bs)) * 64)
    physical = heads * (min(logical, q * width) if cross_query_dedup else q * width)
    rows = q * heads
    return (physical * bs * 384 + 2 * rows * (width + 5) * 4 + rows * groups * 64 * 16
            + logical * heads * 16 + 4 * 1024**2)


class GRSelectedTransport:
    """Plan, fetch and attend one layer's selected blocks for one user."""

    def __init__(self, cache, *, read_order="consumption_depth", cross_query_dedup=True,
                 cuda_graphs=False, capacity=8, workspace_bytes=2 * 1024**3,
                 hot_policy="frequency", spin_limit=1 << 32, query_group=1,
                 async_hot=False, attend_ctas=0):
        if read_order not in _lib.READ_ORDERS:
            raise ValueError("Invalid NSA read priority configuration")
        if hot_policy not in ("frequency", "static", "replica"):
            raise ValueError("hot_policy must be 'frequency', 'static' or 'replica'")
        if query_group != 1:
            raise ValueError("Only single-token consumers (query_group=1) are supported")
        if capacity < 1 or workspace_bytes < 1:
            raise ValueError("Invalid GR selected resource policy")
        if attend_ctas < 0:
            raise ValueError("attend_ctas must be >= 0 (0: every SM)")
        _lib.lib()  # fail loudly now if the extension is missing
        self.cache, self.pool = cache, cache.pool
        self.read_order, self.cross_query_dedup = read_order, cross_query_dedup
        self.hot_policy, self.spin_limit = hot_policy, spin_limit
        # attend_ctas > 0 caps the IO/attention launch at that many CTAs (one
        # per SM), leaving the other SMs to callers that run other work on
        # concurrent streams; the plan's consumer count follows the cap.
        self.attend_ctas = attend_ctas
        adapter = ActivePlanAdapter if cross_query_dedup else QueryPrivatePlanAdapter
        # "replica": residency from the cache's static per-token table
        # (HiSparseCache.enable_replica); like "static", nothing is committed.
        self.active_plan = adapter(cache, read_order=read_order,
                                   residency_table=hot_policy == "replica")
        self.cuda_graphs, self.capacity = cuda_graphs, capacity
        self.workspace_budget = workspace_bytes
        self.workspaces = OrderedDict()
        self.descriptors = OrderedDict()
        self.workspace_allocations = self.workspace_evictions = 0
        self.captures = self.replays = 0
        self.calls = 0
        self.submitted = False
        self.last_done = torch.cuda.Event()
        self.last_stats = {}
        self._capacity_cache = {}
        self._capture_stream = None
        self._graph_refs = []
        # When a list, eager calls append (start, end, workspace) CUDA events
        # bracketing the fetch/attend launch on its stream (bench roofline).
        self.kernel_timing = None
        self.async_hot = async_hot
        self._hot_stream = None
        self._hot_pending = False

    # -- reference surface -----------------------------------------------
    def refusal(self, queries, cached, heads, groups, width, bs):
        """Reason to refuse before any side effect, else None (transport.py:215-237)."""
        if not 1 <= queries <= QUERY_BUCKETS[-1]:
            return "query_bucket_limit"
        if groups != 16 or bs not in (16, 32, 64):
            return "geometry"
        estimate = workspace_estimate(queries, cached, heads, groups, width, bs,
                                      cross_query_dedup=self.cross_query_dedup)
        return "workspace_budget" if estimate > self.workspace_budget else None

    def close(self):
        if self.submitted:
            self.last_done.synchronize()
        for w in self.workspaces.values():
            w.pop("graph", None)
        self.workspaces.clear()

    @property
    def graphs(self):
        return dict(entries=sum("graph" in w for w in self.workspaces.values()),
                    captures=self.captures, replays=self.replays)

    # -- workspace ---------------------------------------------------------
    def _attention_warps(self, bs):
        if bs not in self._capacity_cache:
            value = _lib.c_i32(0)
            _lib.check(_lib.lib().cxs_attend_capacity(bs, value))
            self._capacity_cache[bs] = value.value
        warps = self._capacity_cache[bs]
        return min(warps, 4 * self.attend_ctas) if self.attend_ctas else warps

    def _workspace(self, qb, heads, width, fetches, bs, window_shape, workspace_id=None):
        # Candidate segments place suffix tokens up to cached + len(current_kv).
        logical = max(f["cached_length"] + max(qb, len(f["current_kv"])) for f in fetches)
        map_blocks = max(64, math.ceil(logical / (64 * bs)) * 64)
        key = (qb, heads, width, bs, map_blocks, window_shape, workspace_id)
        if key in self.workspaces:
            self.workspaces.move_to_end(key)
            return self.workspaces[key]
        estimate = workspace_estimate(qb, max(f["cached_length"] for f in fetches), heads, 16,
                                      width, bs, cross_query_dedup=self.cross_query_dedup)
        if estimate > self.workspace_budget:
            raise GRWorkspaceLimit(
                f"GR workspace estimate {estimate} exceeds {self.workspace_budget} bytes")
        resident = sum(w["allocated_bytes"] for w in self.workspaces.values())
        while self.workspaces and (len(self.workspaces) >= self.capacity
                                   or resident + estimate > self.workspace_budget):
            # Least recently used first; a workspace bound into a caller's
            # captured graph stays (its buffers are baked into the graph).
            victim = next((k for k, v in self.workspaces.items() if not v.get("pinned")), None)
            if victim is None:
                raise GRWorkspaceLimit("every cached workspace is bound into a captured graph")
            if torch.cuda.is_current_stream_capturing():
                # Evicting waits for the last launch, which a capture forbids
                # (the wait would invalidate the caller's graph).
                raise GRWorkspaceLimit(
                    "workspace cache full while a graph is being captured: give the transport "
                    "room for every workspace the captured graphs hold (capacity / "
                    "workspace_bytes)")
            if self.submitted:
                self.last_done.synchronize()
            old = self.workspaces.pop(victim)
            old.pop("graph", None)
            resident -= old["allocated_bytes"]
            self.workspace_evictions += 1
        rows = qb * heads
        consumers = min(rows, self._attention_warps(bs))
        device = self.cache.data.device
        w = self.active_plan.allocate(qb, heads, width, fetches, bs, map_blocks=map_blocks,
                                      consumer_ctas=consumers, device=device)
        p = w["physical"]

        def empty(shape, dtype=torch.int32):
            return torch.empty(shape, dtype=dtype, device=device)

        plan_only = isinstance(workspace_id, tuple) and workspace_id[:1] == ("plan_only",)
        staging_blocks = 1 if plan_only else p  # planner-only workspaces move no payload
        w.update(
            query=torch.zeros((qb, heads, 16, 64), dtype=torch.bfloat16, device=device),
            blocks=torch.full((qb, heads, width), -1, dtype=torch.int32, device=device),
            in_positions=torch.full((qb,), -1, dtype=torch.int32, device=device),
            desc=empty((heads, 5), torch.int64),
            kv=torch.zeros((staging_blocks, bs, 128), dtype=torch.bfloat16, device=device),
            sources=empty((p,), torch.int64), kinds=empty((p,)), ready=empty((p,)),
            control=torch.zeros((4,), dtype=torch.int32, device=device),
            error=torch.zeros((1,), dtype=torch.int32, device=device),
            output=torch.zeros((qb, heads, 16, 64), dtype=torch.bfloat16, device=device),
            window_shape=window_shape,
        )
        if window_shape is not None:
            window_len = window_shape[0]
            w.update(
                window_kv=torch.zeros((window_len, heads, 128), dtype=torch.bfloat16,
                                      device=device),
                compressed=torch.zeros((qb, heads, 16, 64), dtype=torch.bfloat16, device=device),
                gates=torch.zeros((qb, heads, 16, 3), dtype=torch.bfloat16, device=device),
            )
        self.active_plan.bind(w, w["blocks"], w["in_positions"], w["desc"],
                              self.pool.region_bases)
        w["binding"] = "static"
        w["c_attend_buffers"] = _lib.AttendBuffers(
            query=w["query"].data_ptr(), kv=w["kv"].data_ptr(),
            all_ids=w["all_ids"].data_ptr(), all_counts=w["all_counts"].data_ptr(),
            row_positions=w["positions"].data_ptr(), starts=w["starts"].data_ptr(),
            valid=w["valid"].data_ptr(), flags=w["flags"].data_ptr(),
            ioids=w["ioids"].data_ptr(), missing=w["missing"].data_ptr(),
            address=w["address"].data_ptr(), sources=w["sources"].data_ptr(),
            kinds=w["kinds"].data_ptr(), ready=w["ready"].data_ptr(),
            control=w["control"].data_ptr(), error=w["error"].data_ptr(),
            window_kv=_lib.ptr(w.get("window_kv")), compressed=_lib.ptr(w.get("compressed")),
            gates=_lib.ptr(w.get("gates")), out=w["output"].data_ptr(),
            first_depth=w["first_depth"].data_ptr(),
            near_consumers=w["near_consumers"].data_ptr())
        w["allocated_bytes"] = sum(v.numel() * v.element_size() for v in w.values()
                                   if isinstance(v, torch.Tensor))
        self.workspaces[key] = w
        self.workspace_allocations += 1
        return w

    def _bind_static(self, w):
        if w.get("binding") == "static":
            return
        self.active_plan.bind(w, w["blocks"], w["in_positions"], w["desc"],
                              self.pool.region_bases)
        for field, key in (("query", "query"), ("window_kv", "window_kv"),
                           ("compressed", "compressed"), ("gates", "gates")):
            setattr(w["c_attend_buffers"], field, _lib.ptr(w.get(key)))
        w["binding"] = "static"

    def _bind_direct(self, w, query, blocks, positions, desc, window_kv, compressed, gates):
        w["c_buffers"].blocks = blocks.data_ptr()
        w["c_buffers"].positions = positions.data_ptr()
        w["c_buffers"].desc = desc.data_ptr()
        b = w["c_attend_buffers"]
        b.query = query.data_ptr()
        b.window_kv = _lib.ptr(window_kv)
        b.compressed = _lib.ptr(compressed)
        b.gates = _lib.ptr(gates)
        w["binding"] = "direct"

    def _execute(self, w, window_start, window, defer_hot=False, segments=(0, 0), output=None):
        stream = torch.cuda.current_stream(self.cache.data.device)
        self.active_plan.plan(w, stream, defer_hot=defer_hot)
        buffers = w["c_attend_buffers"]
        out_heads = out_head0 = 0
        if output is None:
            buffers.out, buffers.out_peer = w["output"].data_ptr(), None
        else:
            local, peer, out_heads, out_head0 = output
            buffers.out, buffers.out_peer = local.data_ptr(), peer
        geometry = _lib.AttendGeometry(
            queries=w["queries"], heads=w["heads"], width=w["width"], block_size=w["bs"],
            physical=w["physical"], window=window if w["window_shape"] else 0,
            window_len=w["window_shape"][0] if w["window_shape"] else 0,
            gate=1 if w["window_shape"] else 0, window_start=window_start,
            spin_limit=self.spin_limit, segment_start=segments[0],
            segment_tokens=segments[1], out_heads=out_heads, out_head0=out_head0,
            ctas=self.attend_ctas)
        timing = self.kernel_timing is not None and not torch.cuda.is_current_stream_capturing()
        if timing:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
        _lib.check(_lib.lib().cxs_fetch_attend(geometry, w["c_attend_buffers"],
                                               stream.cuda_stream))
        if timing:
            end.record(stream)
            self.kernel_timing.append((start, end, w))

    # -- main entry --------------------------------------------------------
    def run(self, query, blocks, positions, fetches, block_size, *, trace=False,
            window=None, window_kv=None, window_start=0, compressed=None, gates=None,
            workspace_id=None, segments=None, output=None):
        """Reference ``run`` plus the fused branches and, optionally, candidate
        segments: ``segments=(segment_start, segment_tokens)`` says that
        ``positions``, ``blocks``, the window buffer and each fetch's
        ``current_kv`` use the candidate-segment layout of
        ``cxs_attend_geometry`` (every candidate sees the history below
        ``segment_start`` and its own suffix only). The plan needs nothing
        else: history blocks deduplicate across candidates, suffix blocks
        stay private to their candidate. ``fetches[h]["cached_length"]`` and
        ``history_length`` must then equal ``segment_start``.

        ``output=(local, peer, out_heads, out_head0)`` routes the attention
        rows of this call's heads into `local` [Q', out_heads, 16, 64] at head
        offset out_head0 and stores the same rows at the device address
        `peer` (a GPU pair's NVLink exchange, ``sharding.PeerExchange``); the
        call then returns `local`."""
        if trace:
            raise ValueError("Collect device activity separately from GR timing")
        segments = tuple(int(x) for x in segments) if segments else (0, 0)
        if output is not None and self.cuda_graphs:
            raise ValueError("an output override needs the caller's own graph capture")
        if segments[1]:
            if (segments[0] % block_size or segments[1] % block_size or segments[0] < 0
                    or segments[1] < 0):
                raise ValueError("segments must be (start, tokens) in whole blocks")
            if any(f["cached_length"] != segments[0] or f["history_length"] != segments[0]
                   for f in fetches):
                raise ValueError("segmented fetches must cache exactly the shared history")
        if (query.ndim != 4 or blocks.ndim != 3 or query.shape[:2] != blocks.shape[:2]
                or len(fetches) != query.shape[1] or positions.shape != (len(query),)
                or blocks.dtype != torch.int32
                or positions.dtype not in (torch.int32, torch.int64)
                or query.shape[2:] != (16, 64) or query.dtype != torch.bfloat16
                or any(t.device != query.device for t in (blocks, positions))):
            raise ValueError("Invalid GR query/selection geometry")
        fused = window is not None
        # A dedicated (per-layer) workspace lets the hot top-k choice and the
        # commit run on a side stream, overlapped with the caller's next work;
        # the caller joins with ``join()`` before the cache is planned again.
        async_hot = (self.async_hot and workspace_id is not None and not self.cuda_graphs
                     and self.hot_policy == "frequency")
        if fused and (window_kv is None or compressed is None or gates is None):
            raise ValueError("Fused branches need window_kv, compressed and gates")
        begin = time.perf_counter_ns()
        device = query.device
        stream = torch.cuda.current_stream(device)
        # Inside a caller's CUDA-graph capture (a whole captured forward) the
        # stream order already serialises calls; events are not recorded.
        capturing = torch.cuda.is_current_stream_capturing()
        if capturing and self.cuda_graphs:
            raise ValueError("cuda_graphs=True cannot nest inside a caller's capture")
        if not capturing:
            if self.submitted:
                stream.wait_event(self.last_done)
            if self.cache.has_last_use:
                stream.wait_event(self.cache.last_use)
        q_count, heads, width = blocks.shape
        qb = query_bucket(q_count)
        window_shape = (len(window_kv), window) if fused else None
        w = self._workspace(qb, heads, width, fetches, block_size, window_shape, workspace_id)
        if capturing:
            w["pinned"] = True  # the caller's graph now holds this workspace's buffers
        # Direct binding: without the transport's own graphs, the kernels read
        # the caller's tensors in place (no staging copies) when they already
        # have the bucket's shape, dtype and layout.
        direct = (not self.cuda_graphs and q_count == qb and query.is_contiguous()
                  and blocks.is_contiguous() and positions.dtype == torch.int32
                  and positions.is_contiguous()
                  and (not fused or (window_kv.is_contiguous() and compressed.is_contiguous()
                                     and gates.is_contiguous()
                                     and window_kv.dtype == torch.bfloat16)))
        layout = tuple((f["row"], f["cached_length"], f["history_length"],
                        f["current_kv"].data_ptr(), len(f["current_kv"])) for f in fetches)
        device_desc = self.descriptors.get(layout)
        if device_desc is None:
            # Uploaded once per layout (transport.py:585-604 caches the same way).
            device_desc = torch.tensor(layout, dtype=torch.int64, pin_memory=True).to(
                device, non_blocking=True)
            self.descriptors[layout] = device_desc
            if len(self.descriptors) > 4096:
                self.descriptors.popitem(last=False)
        else:
            self.descriptors.move_to_end(layout)
        if capturing:
            self._graph_refs.append(device_desc)  # the captured plan reads this buffer
        if direct:
            self._bind_direct(w, query, blocks, positions, device_desc, window_kv, compressed,
                              gates)
        else:
            # Stage inputs into the workspace's static buffers (graph-safe).
            self._bind_static(w)
            w["query"][:q_count].copy_(query)
            w["blocks"][:q_count].copy_(blocks)
            w["in_positions"][:q_count].copy_(positions)
            if q_count < qb:
                w["blocks"][q_count:].fill_(-1)
                w["in_positions"][q_count:].fill_(-1)
            w["desc"].copy_(device_desc, non_blocking=True)
            if fused:
                w["window_kv"].copy_(window_kv)
                w["compressed"][:q_count].copy_(compressed)
                w["gates"][:q_count].copy_(gates)
        for f in fetches:
            f["current_kv"].record_stream(stream)
        if self.cuda_graphs:
            graph_key = (window_start, window, segments)
            if w.get("graph_key") != graph_key:
                w.pop("graph", None)
                self._execute(w, window_start, window, segments=segments)  # warm-up
                graph = torch.cuda.CUDAGraph()
                if self._capture_stream is None:
                    self._capture_stream = torch.cuda.Stream(device)
                self._capture_stream.wait_stream(stream)
                with torch.cuda.graph(graph, stream=self._capture_stream):
                    self._execute(w, window_start, window, segments=segments)
                stream.wait_stream(self._capture_stream)
                w["graph"], w["graph_key"] = graph, graph_key
                self.captures += 1
            w["graph"].replay()
            self.replays += 1
        else:
            self._execute(w, window_start, window, defer_hot=async_hot, segments=segments,
                          output=output)
        if workspace_id is None:
            counters = DeferredLayerCounters(w["stats"].clone(), 1, self.pool.backend,
                                             w["error"].clone())
        else:  # a dedicated workspace: its counters stay valid until its next call
            counters = DeferredLayerCounters(w["stats"], 1, self.pool.backend, w["error"])
        if not capturing:
            self.pool._pending_read_counts.append((w["region_counts"].clone(), 1))
        if async_hot:
            if self._hot_stream is None:
                self._hot_stream = torch.cuda.Stream(device)
            self._hot_stream.wait_stream(stream)
            with torch.cuda.stream(self._hot_stream):
                self.active_plan.select_and_retain_hot(w, w["kv"], self._hot_stream)
            self._hot_pending = True
        elif self.hot_policy == "frequency":
            self.active_plan.retain_hot(w, w["kv"], stream)
        if not capturing:
            self.last_done.record(stream)
            self.cache.last_use.record(stream)
        self.cache.has_last_use = self.submitted = True
        self.cache.planner_calls += 1
        self.calls += 1
        self.last_stats = dict(
            backend=self.pool.backend,
            planner="active_gpu" if self.cross_query_dedup else "query_private_gpu",
            cross_query_dedup=self.cross_query_dedup, read_order=self.read_order,
            effective_q=q_count, query_bucket=qb, history=[f["history_length"] for f in fetches],
            consumer="tma_bounded_rows", consumer_ctas=w["consumer_ctas"],
            io_policy="tma_block_ready", tma_copy="bulk_1d",
            partial_block_policy="external_token_gather", cpu_selection_downloads=0,
            fused_branches=fused, segments=segments, workspace_allocations=self.workspace_allocations,
            workspace_evictions=self.workspace_evictions,
            workspace_bytes=sum(x["allocated_bytes"] for x in self.workspaces.values()),
            logical_block_capacity=w["map_blocks"], active_block_capacity=w["physical"],
            persistent_mapping_bytes=w["persistent_mapping_bytes"],
            total_submit_wall_ms=(time.perf_counter_ns() - begin) / 1e6,
        )
        return (w["output"] if output is None else output[0])[:q_count], counters

    def plan_only(self, query, blocks, positions, fetches, block_size, *, workspace_id=None):
        """Run only the fetch planner on these selections (no IO, attention or
        commit) and return its DeferredLayerCounters: used to compare the
        fetched bytes of the deduplicating and query-private plans."""
        q_count, heads, width = blocks.shape
        qb = query_bucket(q_count)
        w = self._workspace(qb, heads, width, fetches, block_size, None, ("plan_only",))
        layout = tuple((f["row"], f["cached_length"], f["history_length"],
                        f["current_kv"].data_ptr(), len(f["current_kv"])) for f in fetches)
        self._bind_static(w)
        w["blocks"][:q_count].copy_(blocks)
        w["in_positions"][:q_count].copy_(positions)
        if q_count < qb:
            w["blocks"][q_count:].fill_(-1)
            w["in_positions"][q_count:].fill_(-1)
        w["desc"].copy_(torch.tensor(layout, dtype=torch.int64, device=query.device))
        self.active_plan.plan(w, torch.cuda.current_stream(query.device), defer_hot=True)
        return DeferredLayerCounters(w["stats"].clone(), 1, self.pool.backend)

    def join(self, stream=None):
        """Make ``stream`` (current by default) wait for side-stream hot commits."""
        if self._hot_pending:
            stream = stream or torch.cuda.current_stream(self.cache.data.device)
            stream.wait_stream(self._hot_stream)
            self._hot_pending = False
            if not torch.cuda.is_current_stream_capturing():
                self.last_done.record(stream)
                self.cache.last_use.record(stream)

    def workspace(self):
        """The most recently used workspace (inspection helper for tests)."""
        return next(reversed(self.workspaces.values()))
