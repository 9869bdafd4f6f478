"""Residency table on the device: the planner resolves history tokens
through `hbm_locs[row, token]` (an HBM replica of any size and pattern)
bit-exactly as the oracle does, and the transport attends over blocks whose
tokens come partly from the replica and partly from the pool."""

from types import SimpleNamespace

import numpy as np
import pytest
import torch

from cxlsparse_b200 import planning
from cxlsparse_b200.mempool import HiSparseCache, MemoryPool
from cxlsparse_b200.transport import GRSelectedTransport
from golden_io import EXACT_KEYS, load, oracle_args, plan_fixtures
from oracle import attention as A
from oracle import plan as P

pytestmark = pytest.mark.gpu


def _pattern(rows, max_history, bs, seed):
    """Seeded residency: the most recent half of the history plus, elsewhere,
    blocks with only their first or second half resident."""
    rng = np.random.default_rng(seed)
    table = np.full((rows, max_history), -1, np.int64)
    slot = 0
    for r in range(rows):
        for b in range(-(-max_history // bs)):
            lo, hi = b * bs, min(max_history, (b + 1) * bs)
            choice = rng.integers(0, 4)
            tokens = {0: range(0), 1: range(lo, hi), 2: range(lo, lo + bs // 2),
                      3: range(lo + bs // 2, hi)}[int(choice)]
            for t in tokens:
                if t < max_history:
                    table[r, t] = slot
                    slot += 1
    return table


@pytest.mark.parametrize("single_launch", [True, False], ids=["fused", "per_phase"])
@pytest.mark.parametrize("path", plan_fixtures(), ids=lambda p: p.stem)
def test_device_plan_with_residency_table_matches_oracle(cuda, path, single_launch):
    z = load(path)
    args = oracle_args(z)
    private = bool(int(z["private"]))
    rows, max_history = args["host_locs"].shape
    table = _pattern(rows, max_history, args["bs"], seed=len(path.stem))
    ref = (P.private_plan if private else P.active_plan)(**args, hbm_locs=table)
    host_locs = torch.from_numpy(z["host_locs"]).to(cuda)
    pool = SimpleNamespace(region_count=len(z["bases"]), page_size=int(z["page_size"]),
                           pool_tokens=int(z["pool_tokens"]))
    cache = SimpleNamespace(
        hot=int(z["hot"]), pool=pool, tags=torch.from_numpy(z["tags"]).to(cuda, torch.int32),
        locs=torch.from_numpy(z["locs"]).to(cuda, torch.int32), host_locs=host_locs,
        max_history=max_history, data=torch.empty(1, device=cuda),
        replica=torch.empty(1, device=cuda),
        replica_locs=torch.from_numpy(table).to(cuda, torch.int32))
    cls = planning.QueryPrivatePlanAdapter if private else planning.ActivePlanAdapter
    adapter = cls(cache, read_order=str(z["read_order"]), residency_table=True)
    blocks = torch.from_numpy(z["blocks"]).to(cuda, torch.int32)
    q, h, width = blocks.shape
    desc = torch.from_numpy(z["desc"]).to(cuda)
    fetches = [dict(cached_length=int(d[1]), current_kv=range(int(d[4]))) for d in z["desc"]]
    w = adapter.allocate(q, h, width, fetches, int(z["bs"]), map_blocks=int(z["map_blocks"]),
                         consumer_ctas=int(z["consumer_ctas"]), device=cuda)
    positions = torch.from_numpy(z["positions"]).to(cuda, torch.int32)
    bases = torch.from_numpy(z["bases"]).to(cuda)
    buffers = adapter.bind(w, blocks, positions, desc, bases)
    buffers.hot_data = int(z["hot_data"])  # addresses are computed, never dereferenced
    if not single_launch:
        w["c_geometry"].launch_mode = 1
    for key in ("address", "hbm", "slots", "valid", "all_ids"):
        w[key].fill_(77)
    adapter.plan(w)
    torch.cuda.synchronize()
    cpu = {k: v.cpu().numpy() for k, v in w.items() if isinstance(v, torch.Tensor)}
    for key in EXACT_KEYS:
        assert np.array_equal(cpu[key].astype(np.int64), np.asarray(ref[key]).astype(np.int64)), key
    missing = int(ref["missing"])
    assert int(cpu["missing"][0]) == missing
    assert np.array_equal(cpu["ioids"][:missing], ref["ioids"][:missing])
    assert ref["stats"][:, 2].sum() > 0 and ref["stats"][:, 3].sum() > 0 or \
        ref["stats"][:, 1].sum() == 0


@pytest.mark.parametrize("read_order", ["physical", "consumption_depth"])
def test_transport_over_partly_resident_blocks(cuda, read_order):
    """Live pool + replica: 67 history tokens per head, BS 16, blocks 0-1
    fully resident, block 2 half resident (tokens 40-47), block 3 cold,
    block 4 (tail) cold history + suffix. Output vs the FP64 oracle; pool
    reads = exactly the non-resident required history tokens."""
    pool = MemoryPool(8, 128, "host", page_size=64)
    try:
        cache = HiSparseCache(pool, rows=2, max_history=256, hot=64, topk=64, dim=128)
        cache.enable_replica(2 * 67)
        g = torch.Generator().manual_seed(31)
        backing = torch.randn(80, 2, 128, generator=g).bfloat16()
        query = torch.randn(13, 2, 16, 64, generator=g).bfloat16().cuda()
        positions = torch.arange(67, 80, device=cuda)
        blocks = torch.tensor([[[0, 1, 2, 4], [3, 2, 1, 4]]] * 13, dtype=torch.int32,
                              device=cuda)
        resident = list(range(32)) + list(range(40, 48))
        fetches = []
        for head in range(2):
            pages = pool.allocate(2)
            slots = pool.token_slots(pages, 0, 67)
            pool.write_many(slots, backing[:67, head].contiguous().cuda())
            cache.bind(head, slots)
            tokens = torch.tensor(resident, device=cuda)
            cache.replicate(head, tokens, backing[resident, head].cuda())
            fetches.append(dict(row=head, cached_length=67, history_length=67,
                                current_kv=backing[67:, head].contiguous().cuda(), pages=pages))
        transport = GRSelectedTransport(cache, hot_policy="replica", read_order=read_order)
        try:
            out, counters = transport.run(query, blocks, positions, fetches, 16)
            torch.cuda.synchronize()
            rows = counters.materialize()
            expected = A.selected_attention(query.cpu(), backing, blocks.cpu(), positions.cpu(),
                                            16)
            torch.testing.assert_close(out.cpu().double(), expected, rtol=0.03, atol=0.03)
            w = transport.workspace()
            kinds = w["kinds"].cpu().numpy()
            flags = w["flags"].cpu().numpy()
            for h in range(2):
                keys = w["active_keys"][h, : int(w["active_counts"][h])].tolist()
                by_block = {b: h * w["per_head"] + i for i, b in enumerate(keys)}
                if 2 in by_block:
                    assert flags[by_block[2]] == 1 and kinds[by_block[2]] == 2  # mixed
                if 0 in by_block:
                    assert flags[by_block[0]] == 0                              # resident
            # Head 0 selects blocks 0,1,2,4: cold = tokens 32-39 and 48-63 of
            # blocks 2 and 4 (the tail block 4 holds history 64-66).
            assert rows[0]["misses"] == 8 + 3
            assert rows[1]["misses"] == 8 + 16 + 3  # blocks 2, 3 and 4
            assert rows[0]["hits"] == 32 + 8
        finally:
            transport.close()
    finally:
        pool.close()


def test_model_with_replica_matches_frequency_policy(cuda):
    """The same model with a static replica (recent blocks + half-resident
    straddling blocks) instead of the frequency hot set reads the same KV
    values from other tiers: its extend is bit-identical (each row takes its
    selected blocks by the plan's read-order key, which does not depend on
    residency), and its pool reads are exactly the selected non-resident
    history tokens."""
    from cxlsparse_b200.model import NSAConfig, NSAExtendModel, residency_pattern

    cfg = NSAConfig(layers=2, hot=64)
    history, extend = 1000, 64
    g = torch.Generator().manual_seed(17)
    tokens = torch.randint(0, cfg.vocab, (history,), generator=g).to(cuda)
    ids = torch.randint(0, cfg.vocab, (extend,), generator=g).to(cuda)
    outs, models = [], []
    try:
        for policy in ("frequency", "replica"):
            model = NSAExtendModel(cfg, device=cuda, seed=0, max_history=history + extend,
                                   chunk=512, hot_policy=policy, replica_blocks=4,
                                   straddle=0.3)
            models.append(model)
            model.prefill(tokens)
            model.prepare_fast(extend)
            outs.append(model.extend_fast(ids).clone())
            torch.cuda.synchronize()
        assert torch.equal(outs[0], outs[1])
        model = models[1]
        resident = residency_pattern(history, cfg.block_size, 4, 0.3, seed=0)
        assert 0 < int(resident.sum()) < history
        for index, counters in enumerate(model.counters):
            rows = counters.materialize()
            w = model.transport.workspaces[next(k for k in model.transport.workspaces
                                                if k[-1] == index)]
            for h in range(model.kv_local):
                keys = w["active_keys"][h, : int(w["active_counts"][h])].cpu()
                req = w["required"][h, : len(keys)].cpu()
                cold = sum(int((~resident[b * 64: b * 64 + min(int(r), history - b * 64)]).sum())
                           for b, r in zip(keys.tolist(), req.tolist()) if b * 64 < history)
                assert rows[h]["misses"] == cold
    finally:
        for model in models:
            model.close()
