"""Host-side transport logic that needs no GPU."""

from types import SimpleNamespace

import pytest
import torch

from cxlsparse_b200 import planning, transport


def _adapter(hot=256, private=False):
    cls = planning.QueryPrivatePlanAdapter if private else planning.ActivePlanAdapter
    return cls(SimpleNamespace(hot=hot, pool=SimpleNamespace(region_count=1)))


@pytest.mark.parametrize("q", [64, 128, 256, 512, 1024])
def test_geometry_capacity_never_truncates_union(q):
    """tests/test_nsa_active_plan.py:118-128."""
    f = dict(cached_length=65536, current_kv=range(q))
    geom = _adapter().geometry(q, 2, 4, [f, f], 16, map_blocks=4160)
    assert geom["per_head"] == min(4160, q * 4)
    assert geom["physical"] == geom["per_head"] * 2
    assert geom["sort_extent"] >= 256


def test_history_buckets_and_truncation_refusal():
    """tests/test_nsa_active_plan.py:131-144 (map_blocks grows with history)."""
    observed = []
    for history in (4096, 8192, 16384, 32768, 65536):
        logical = history + 64
        map_blocks = max(64, -(-logical // (64 * 16)) * 64)
        fetch = dict(cached_length=history, current_kv=range(64))
        observed.append(_adapter().geometry(64, 2, 4, [fetch] * 2, 16, map_blocks=map_blocks))
    assert all(g["per_head"] == 256 for g in observed)
    assert [g["map_blocks"] for g in observed] == [320, 576, 1088, 2112, 4160]
    fetch = dict(cached_length=4096, current_kv=range(64))
    with pytest.raises(ValueError, match="truncate"):
        _adapter().geometry(64, 2, 4, [fetch] * 2, 16, map_blocks=256)


def test_private_capacity_is_not_limited_by_history_union():
    """tests/test_nsa_query_private_plan.py:12-25."""
    fetch = dict(cached_length=4096, current_kv=range(128))
    w = _adapter(private=True).geometry(128, 2, 16, [fetch, fetch], 16)
    assert w["per_head"] == 128 * 16 and w["physical"] == 128 * 16 * 2
    assert w["sort_extent"] == 4096 + 128


def test_query_buckets():
    assert [transport.query_bucket(n) for n in (1, 64, 65, 1024, 1025)] == \
        [64, 64, 128, 1024, 2048]
    with pytest.raises(transport.GRWorkspaceLimit):
        transport.query_bucket(5000)
    with pytest.raises(ValueError):
        transport.query_bucket(0)


def test_deferred_counters_materialize_and_errors():
    stats = torch.tensor([[24, 19, 4, 15, 38, 6, 0], [3, 2, 0, 2, 5, 1, 0]])
    rows = transport.DeferredLayerCounters(stats, 1).materialize()
    assert rows[0]["misses"] == 15 and rows[0]["deduplicated_references"] == 38 - 19
    assert rows[0]["h2d_transfers"] == 1 and rows[1]["h2d_transfers"] == 0
    bad = stats.clone()
    bad[1, 6] = 1
    with pytest.raises(ValueError):
        transport.DeferredLayerCounters(bad, 1).materialize()
    with pytest.raises(RuntimeError, match="device error"):
        transport.DeferredLayerCounters(stats, 1, device_error=torch.tensor([1])).materialize()


def test_workspace_estimate_budget_refusal():
    assert transport.workspace_estimate(256, 16384, 2, 16, 16, 64) < 2 * 1024**3
    t = transport.GRSelectedTransport.__new__(transport.GRSelectedTransport)
    t.workspace_budget, t.cross_query_dedup = 1024, True
    assert t.refusal(256, 16384, 2, 16, 16, 64) == "workspace_budget"
    assert t.refusal(5000, 16384, 2, 16, 16, 64) == "query_bucket_limit"
    assert t.refusal(256, 16384, 2, 8, 16, 64) == "geometry"


def test_attend_cta_cap_sets_the_plan_consumer_count():
    """attend_ctas caps the attention launch; the planner's consumer count
    (attention warps, 4 per CTA) follows the cap and never exceeds what one
    CTA per SM gives. A negative cap is refused before touching the device."""
    with pytest.raises(ValueError, match="attend_ctas"):
        transport.GRSelectedTransport(SimpleNamespace(pool=None), attend_ctas=-1)
    t = transport.GRSelectedTransport.__new__(transport.GRSelectedTransport)
    t._capacity_cache = {64: 148 * 4}
    for cap, warps in ((0, 592), (37, 148), (1, 4), (148, 592), (500, 592)):
        t.attend_ctas = cap
        assert t._attention_warps(64) == warps, cap
