"""Device planner (cxs_plan through the C ABI) vs the reference's own plans.

Each fixture was produced by running the reference planner; the device plan
must reproduce every array bit-exactly (dedup tables, compact layout, source
addresses, stats, occurrence rows, consumption order, hot choice). Addresses
in the fixtures are plain integers: the planner computes them but never
dereferences them.
"""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from cxlsparse_b200 import planning
from golden_io import EXACT_KEYS, load, oracle_args, plan_fixtures
from oracle import plan as P

pytestmark = pytest.mark.gpu


def run_device_plan(z, device, *, private=None, read_order=None, consumer_ctas=None,
                    single_launch=True):
    private = bool(int(z["private"])) if private is None else private
    read_order = read_order or str(z["read_order"])
    tags = torch.from_numpy(z["tags"]).to(device, torch.int32)
    locs = torch.from_numpy(z["locs"]).to(device, torch.int32)
    host_locs = torch.from_numpy(z["host_locs"]).to(device)
    hot = int(z["hot"])
    pool = SimpleNamespace(region_count=len(z["bases"]), page_size=int(z["page_size"]),
                           pool_tokens=int(z["pool_tokens"]))
    cache = SimpleNamespace(hot=hot, pool=pool, tags=tags, locs=locs, host_locs=host_locs,
                            max_history=host_locs.shape[1],
                            data=torch.empty(1, device=device))
    cls = planning.QueryPrivatePlanAdapter if private else planning.ActivePlanAdapter
    adapter = cls(cache, read_order=read_order)
    blocks = torch.from_numpy(z["blocks"]).to(device, torch.int32)
    q, h, width = blocks.shape
    desc = torch.from_numpy(z["desc"]).to(device)
    fetches = [dict(cached_length=int(d[1]), current_kv=range(int(d[4]))) for d in z["desc"]]
    w = adapter.allocate(q, h, width, fetches, int(z["bs"]), map_blocks=int(z["map_blocks"]),
                         consumer_ctas=consumer_ctas or int(z["consumer_ctas"]), device=device)
    positions = torch.from_numpy(z["positions"]).to(device, torch.int32)
    bases = torch.from_numpy(z["bases"]).to(device)
    buffers = adapter.bind(w, blocks, positions, desc, bases)
    # The plan reads these on every (graph) replay: keep them alive with w.
    w["_inputs"] = (blocks, positions, desc, bases, tags, locs, host_locs, cache)
    buffers.hot_data = int(z["hot_data"])
    if not single_launch:
        w["c_geometry"].launch_mode = 1  # one launch per planner phase
    # Stale scratch from an earlier call must not leak into the next plan.
    for key in ("address", "hbm", "slots", "valid", "all_ids", "chosen"):
        w[key].fill_(77)
    adapter.plan(w)
    torch.cuda.synchronize()
    return w


@pytest.mark.parametrize("single_launch", [True, False], ids=["fused", "per_phase"])
@pytest.mark.parametrize("path", plan_fixtures(), ids=lambda p: p.stem)
def test_device_plan_matches_reference_bit_exact(cuda, path, single_launch):
    z = load(path)
    w = run_device_plan(z, cuda, single_launch=single_launch)
    cpu = {k: v.cpu().numpy() for k, v in w.items() if isinstance(v, torch.Tensor)}
    for key in EXACT_KEYS:
        assert np.array_equal(cpu[key].astype(np.int64), z["ref_" + key].astype(np.int64)), key
    for h, count in enumerate(cpu["active_counts"]):
        assert np.array_equal(cpu["active_keys"][h, :count], z["ref_active_keys"][h, :count])
    missing = int(cpu["missing"][0])
    assert missing == int(z["ref_missing"][0])
    assert np.array_equal(cpu["ioids"][:missing], z["ref_ioids"][:missing])
    assert (cpu["ioids"][missing:] == -1).all()
    flags = cpu["flags"].astype(bool)
    assert np.array_equal(cpu["ranks"][flags], z["ref_ranks"][flags])
    assert (cpu["ranks"][~flags] == -1).all()
    hot = int(z["hot"])
    assert np.array_equal(cpu["chosen"], z["chosen"][:, :hot].astype(np.int64))


@pytest.mark.parametrize("single_launch", [True, False], ids=["fused", "per_phase"])
@pytest.mark.parametrize("order", ["physical", "consumption_depth", "consumption_depth_shared"])
@pytest.mark.parametrize("consumers", [1, 3, 256])
def test_device_read_orders_match_oracle(cuda, order, consumers, single_launch):
    z = load(plan_fixtures()[3])  # miss_bs64_shared_regions
    w = run_device_plan(z, cuda, read_order=order, consumer_ctas=consumers,
                        single_launch=single_launch)
    args = oracle_args(z)
    args.update(read_order=order, consumer_ctas=min(consumers, w["rows"]))
    ref = P.active_plan(**args)
    missing = int(ref["missing"])
    assert int(w["missing"].item()) == missing
    assert np.array_equal(w["ioids"].cpu().numpy()[:missing], ref["ioids"][:missing])
    if order != "physical":
        flags = ref["flags"].astype(bool)
        assert np.array_equal(w["first_depth"].cpu().numpy()[flags], ref["first_depth"][flags])
    if order == "consumption_depth_shared":
        flags = ref["flags"].astype(bool)
        assert np.array_equal(w["near_consumers"].cpu().numpy()[flags], ref["near"][flags])


def test_device_plan_replays_in_a_cuda_graph(cuda):
    z = load(plan_fixtures()[2])  # miss_bs16_depth
    w = run_device_plan(z, cuda)
    expected = {k: w[k].clone() for k in ("stats", "all_ids", "ioids", "address", "chosen")}
    adapter_stream = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    from cxlsparse_b200 import _lib
    with torch.cuda.graph(graph, stream=adapter_stream):
        _lib.check(_lib.lib().cxs_plan(w["c_geometry"], w["c_buffers"],
                                       torch.cuda.current_stream().cuda_stream))
    for _ in range(3):
        w["all_ids"].fill_(5)
        w["stats"].fill_(9)
        graph.replay()
        torch.cuda.synchronize()
        for key, value in expected.items():
            assert torch.equal(w[key], value), key


def test_large_private_plan_physical_publish(cuda):
    """Plans beyond one publish CTA (P > 16384) use the chunked compaction."""
    from cxlsparse_b200.mempool import HiSparseCache, MemoryPool

    pool = MemoryPool(16 * 2 + 8, 128, page_size=64)
    try:
        cache = HiSparseCache(pool, rows=2, max_history=1024 + 1100, hot=64, topk=64)
        for h in range(2):
            cache.bind(h, pool.token_slots(pool.allocate(16), 0, 1024))
        adapter = planning.QueryPrivatePlanAdapter(cache, read_order="physical")
        g = torch.Generator().manual_seed(5)
        q = 1100
        positions = torch.arange(1024, 1024 + q, dtype=torch.int32)
        blocks = torch.randint(0, 16, (q, 2, 16), generator=g, dtype=torch.int32)
        fetches = [dict(row=h, cached_length=1024, history_length=1024,
                        current_kv=torch.empty(q, 128, device=cuda)) for h in range(2)]
        w = adapter.allocate(q, 2, 16, fetches, 64, device=cuda)
        assert w["physical"] > 16384
        desc = torch.tensor([(h, 1024, 1024, 1 << 40, q) for h in range(2)], device=cuda)
        blocks_d, positions_d = blocks.to(cuda), positions.to(cuda)
        adapter.bind(w, blocks_d, positions_d, desc, pool.region_bases)
        w["_inputs"] = (blocks_d, positions_d, desc)
        adapter.plan(w)
        torch.cuda.synchronize()
        flags = w["flags"].cpu().numpy()
        ioids, ranks, missing = P.physical_order(flags)
        assert int(w["missing"].item()) == missing > 16384
        assert np.array_equal(w["ioids"].cpu().numpy()[:missing], ioids[:missing])
        assert np.array_equal(w["ranks"].cpu().numpy()[flags.astype(bool)],
                              ranks[flags.astype(bool)])
        assert int(w["stats"][:, 3].sum()) == sum(int(v) for v in w["valid"].cpu().numpy()
                                                  [flags.astype(bool)])
    finally:
        pool.close()
