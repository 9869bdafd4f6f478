"""Fetch-planner adapters over the C ABI (``cxs_plan`` / ``cxs_plan_commit_hot``).

Mirrors ``cxl_recsys/models/nsa/planning/active.py:503-925``
(``ActivePlanAdapter``) and ``planning/query_private.py:219-475``
(``QueryPrivatePlanAdapter``): same geometry rules, same workspace array
names and layouts, so a reference-style caller (or test) can inspect any
intermediate. Planning never downloads data to the host and is graph-capturable.
"""

import math

import torch

from . import _lib


def next_pow2(x):
    return 1 << max(0, int(x) - 1).bit_length()


class ActivePlanAdapter:
    """Deduplicating plan: identical (head, block) requests share one slot."""

    private = False

    def __init__(self, cache, *, read_order="consumption_depth", residency_table=False):
        if read_order not in _lib.READ_ORDERS:
            raise ValueError("Invalid NSA read priority configuration")
        if cache.hot < 1:
            raise ValueError("Positive hot capacity is required")
        if residency_table and cache.replica_locs is None:
            raise ValueError("residency_table needs cache.enable_replica()")
        self.cache, self.pool = cache, cache.pool
        self.read_order = read_order
        # True: residency from the cache's per-token table (cache.replica /
        # replica_locs) instead of the hot tags.
        self.residency_table = residency_table

    # planning/active.py:517-552
    def geometry(self, queries, heads, width, fetches, bs, *, map_blocks=None):
        if bs < 1 or bs & (bs - 1) or not heads or not width or not queries:
            raise ValueError("Nonempty geometry and a power-of-two block size required")
        if len(fetches) != heads:
            raise ValueError("Selected geometry does not match fetch descriptors")
        needed = math.ceil(max(f["cached_length"] + len(f["current_kv"]) for f in fetches) / bs)
        if map_blocks is None:
            map_blocks = needed
        if map_blocks < needed or map_blocks < 1:
            raise ValueError("History mapping capacity cannot truncate a request")
        if map_blocks * bs > 2**31 - 1:
            raise ValueError("Absolute token addressing must fit int32")
        per_head = self._per_head(queries, width, map_blocks)
        return dict(
            heads=heads, width=width, bs=bs, queries=queries, rows=queries * heads,
            map_blocks=map_blocks, per_head=per_head, physical=heads * per_head,
            sort_extent=self._sort_extent(per_head, map_blocks, bs),
            hash_capacity=next_pow2(2 * self.cache.hot),
        )

    def _per_head(self, queries, width, map_blocks):
        return min(map_blocks, queries * width)

    def _sort_extent(self, per_head, map_blocks, bs):
        return max(per_head * bs, self.cache.hot)

    def allocate(self, queries, heads, width, fetches, bs, *, map_blocks=None,
                 consumer_ctas=None, device=None):
        w = self.geometry(queries, heads, width, fetches, bs, map_blocks=map_blocks)
        device = device or self.cache.data.device
        h, c, p, rows = w["heads"], w["per_head"], w["physical"], w["rows"]

        def empty(shape, dtype=torch.int32, fill=None):
            t = torch.empty(shape, dtype=dtype, device=device)
            if fill is not None:
                t.fill_(fill)
            return t

        mapping_shape = (h, c) if self.private else (h, w["map_blocks"] + 1)
        w.update(
            mapping=empty(mapping_shape, fill=-1),
            insert_keys=empty((h, c)),
            active_keys=empty((h, c), fill=2**31 - 1),
            active_counts=empty((h,)),
            required=empty((h, c)),
            frequencies=empty((h, w["sort_extent"])),
            stats=empty((h, 7)),
            address=empty((p, bs), torch.int64),
            hbm=empty((p, bs), torch.int64),
            valid=empty((p,)),
            starts=empty((p,)),
            flags=empty((p,)),
            slots=empty((p * bs,), torch.int64),
            ioids=empty((p,)),
            ranks=empty((p,)),
            missing=empty((1,)),
            all_ids=empty((rows, width)),
            all_counts=empty((rows,)),
            positions=empty((rows,)),
            region_counts=empty((self.pool.region_count,)),
            row_depth=empty((rows,)),
            first_depth=empty((p,)),
            near_consumers=empty((p,)),
            chosen=empty((h, self.cache.hot)),
        )
        if self.private:
            w.update(
                private_required=empty((h, c)),
                private_occurrences=empty((rows, width)),
                canonical=empty((h, w["sort_extent"])),
            )
        w["consumer_ctas"] = max(1, min(rows, consumer_ctas or 256))
        w["read_order"] = self.read_order
        w["c_geometry"] = _lib.PlanGeometry(
            queries=queries, heads=h, width=width, block_size=bs,
            map_blocks=w["map_blocks"], per_head=c, sort_extent=w["sort_extent"],
            hot=self.cache.hot, max_history=self.cache.max_history,
            regions=self.pool.region_count, page_size=self.pool.page_size,
            consumer_ctas=w["consumer_ctas"], read_order=_lib.READ_ORDERS[self.read_order],
            private_plan=int(self.private), pool_tokens=self.pool.pool_tokens)
        _lib.check(_lib.lib().cxs_plan_check(w["c_geometry"]))
        w["scratch_bytes"] = sum(v.numel() * v.element_size() for k, v in w.items()
                                 if isinstance(v, torch.Tensor) and k != "mapping")
        w["persistent_mapping_bytes"] = w["mapping"].numel() * 4
        return w

    def bind(self, w, blocks, positions, desc, bases):
        """Fill the C buffer table for these (static) input tensors."""
        table = self.residency_table
        names = dict(
            blocks=blocks, positions=positions, desc=desc, bases=bases,
            tags=self.cache.tags, locs=self.cache.locs, host_locs=self.cache.host_locs,
            hot_data=self.cache.replica if table else self.cache.data,
            hbm_locs=self.cache.replica_locs if table else None,
            row_positions=w["positions"])
        fields = {}
        for field in _lib.PLAN_BUFFER_FIELDS:
            tensor = names.get(field, w.get(field))
            fields[field] = None if tensor is None else tensor.data_ptr()
        w["c_buffers"] = _lib.PlanBuffers(**fields)
        return w["c_buffers"]

    def plan(self, w, stream=None, *, defer_hot=False):
        """Enqueue the plan on ``stream`` (current stream by default).

        ``defer_hot`` leaves the hot top-k choice to ``select_and_retain_hot``.
        """
        stream = stream or torch.cuda.current_stream(self.cache.data.device)
        fn = _lib.lib().cxs_plan_core if defer_hot else _lib.lib().cxs_plan
        _lib.check(fn(w["c_geometry"], w["c_buffers"], stream.cuda_stream))
        return w["chosen"]

    def select_and_retain_hot(self, w, kv, stream=None):
        """Hot top-k choice + commit (after ``plan(defer_hot=True)`` and attention)."""
        stream = stream or torch.cuda.current_stream(self.cache.data.device)
        _lib.check(_lib.lib().cxs_plan_select_commit_hot(
            w["c_geometry"], w["c_buffers"], kv.data_ptr(), self.cache.tags.data_ptr(),
            self.cache.data.data_ptr(), stream.cuda_stream))

    def retain_hot(self, w, kv, stream=None):
        """Commit the chosen hot tokens after attention (active.py:909-925)."""
        stream = stream or torch.cuda.current_stream(self.cache.data.device)
        _lib.check(_lib.lib().cxs_plan_commit_hot(
            w["c_geometry"], w["c_buffers"], kv.data_ptr(), self.cache.tags.data_ptr(),
            self.cache.data.data_ptr(), stream.cuda_stream))


class QueryPrivatePlanAdapter(ActivePlanAdapter):
    """No cross-row sharing: each (row, head, block) owns its payload slot."""

    private = True

    def _per_head(self, queries, width, map_blocks):
        return queries * width

    def _sort_extent(self, per_head, map_blocks, bs):
        return max(map_blocks * bs, self.cache.hot)
