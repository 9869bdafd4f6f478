"""The workspace budget check rests on workspace_estimate being an upper
bound: the transport refuses (GRWorkspaceLimit) before any allocation when
the estimate exceeds the budget, so the estimate must never undercount what
a workspace then allocates. Checked on the meta device (no memory, no GPU)
by building real transport workspaces at the benchmark shapes: one
candidate, candidate segments, the KV-head split's long history, the dedup
stress size, query-private plans and smaller blocks."""

from collections import OrderedDict
from types import SimpleNamespace

import pytest
import torch

from cxlsparse_b200 import planning, transport
from cxlsparse_b200.segments import SegmentLayout

META = torch.device("meta")


def _transport(dedup, hot=256, max_history=140000):
    pool = SimpleNamespace(region_count=1, page_size=64, pool_tokens=1 << 26, backend="host",
                           region_bases=torch.zeros(1, dtype=torch.int64, device=META))
    empty = torch.empty(0, device=META)
    cache = SimpleNamespace(hot=hot, max_history=max_history, pool=pool, data=empty,
                            tags=empty, locs=empty, host_locs=empty, replica=None,
                            replica_locs=None)
    t = transport.GRSelectedTransport.__new__(transport.GRSelectedTransport)
    t.cache, t.pool, t.cross_query_dedup = cache, pool, dedup
    adapter = planning.ActivePlanAdapter if dedup else planning.QueryPrivatePlanAdapter
    t.active_plan = adapter(cache, read_order="consumption_depth")
    t.workspaces, t.capacity, t.workspace_budget = OrderedDict(), 8, 1 << 50
    t.submitted, t.workspace_allocations, t.workspace_evictions = False, 0, 0
    t._capacity_cache, t.attend_ctas = {16: 592, 32: 592, 64: 592}, 0
    return t


CASES = [
    # history, extend per candidate, candidates, heads, width, bs, dedup
    (16384, 256, 1, 2, 16, 64, True),      # headline
    (4096, 128, 1, 2, 16, 64, True),
    (16384, 128, 16, 2, 16, 64, True),     # dedup stress, candidate segments
    (33791, 256, 4, 2, 16, 64, True),      # serving, partial tail block
    (131072, 256, 8, 1, 16, 64, True),     # KV-head split: one head per GPU
    (1000, 64, 3, 2, 16, 16, True),
    (777, 64, 2, 2, 8, 32, True),
    (900, 24, 1, 2, 8, 64, False),         # query-private plan
    (1500, 64, 2, 2, 16, 16, False),
]


@pytest.mark.parametrize("history,extend,candidates,heads,width,bs,dedup", CASES)
def test_estimate_bounds_the_allocated_workspace(history, extend, candidates, heads, width,
                                                 bs, dedup):
    t = _transport(dedup)
    rows = extend * candidates
    if candidates == 1:
        cached, suffix, window_len = history, extend, 511 + extend
    else:
        layout = SegmentLayout(history, extend, candidates, bs)
        cached, suffix = layout.start, candidates * layout.tokens
        window_len = 511 + suffix
    fetches = [dict(row=h, cached_length=cached, history_length=cached,
                    current_kv=torch.empty(suffix, 128, device=META)) for h in range(heads)]
    qb = transport.query_bucket(rows)
    w = t._workspace(qb, heads, width, fetches, bs, (window_len, 512), workspace_id=0)
    estimate = transport.workspace_estimate(qb, cached, heads, 16, width, bs,
                                            cross_query_dedup=dedup)
    assert w["allocated_bytes"] <= estimate, (w["allocated_bytes"], estimate)
