"""End-to-end selected transport: live mapped-host pool, mixed tiers, oracles.

Restates the reference's TMA transport tests (tests/test_nsa_tma_transport.py,
tests/test_nsa_dependency_order.py:260-319) on the B200 kernels: output vs the
FP64 oracle at rtol = atol = 0.03, exact pool read bytes (misses x 256), hot
commit byte-exact, poisoned staging / stale ready flags, graph replay and
read-order invariance.
"""

import pytest
import torch

from cxlsparse_b200.transport import GRSelectedTransport
from nsa_case import setup_case
from oracle.attention import selected_attention

pytestmark = pytest.mark.gpu


def _oracle(query, backing, blocks, positions):
    return selected_attention(query.cpu(), backing, blocks.cpu(), positions.cpu(), 16)


@pytest.mark.parametrize("residency", ["miss", "partial", "hit", "empty"])
def test_live_sources_long_queries_and_replay(cuda, residency):
    pool, cache, backing, source_q, source_pos, source_blocks, fetches = setup_case(residency)
    transport = GRSelectedTransport(cache, hot_policy="static")
    try:
        for length in (13, 129, 769):
            index = torch.arange(length, device="cuda") % len(source_q)
            query = source_q[index].contiguous()
            positions = source_pos[index].contiguous()
            blocks = source_blocks[index].contiguous()
            for replay in range(2):
                if replay:
                    query.mul_(-0.75)
                    backing[67:].add_(0.25)
                    for head, fetch in enumerate(fetches):
                        fetch["current_kv"].copy_(backing[67:, head])
                expected = _oracle(query, backing, blocks, positions)
                before = pool.read_bytes
                output, counters = transport.run(query, blocks, positions, fetches, 16)
                transport.last_done.synchronize()
                rows = counters.materialize()
                pool.flush_read_stats()
                torch.testing.assert_close(output.cpu().double(), expected, rtol=0.03, atol=0.03)
                assert pool.read_bytes - before == sum(r["misses"] for r in rows) * 256
                assert transport.last_stats["effective_q"] == length
                if length == 13 and replay == 0:
                    kinds = transport.workspace()["kinds"].cpu().tolist()
                    if residency == "miss":
                        assert 1 in kinds and 2 in kinds
                    elif residency == "partial":
                        assert 2 in kinds
                    else:
                        assert set(kinds) <= {0}
                    if residency != "empty":
                        assert sum(r["old_references"] for r in rows) == 13 * (3 * 16 + 3) * 2
    finally:
        transport.close()
        pool.close()


@pytest.mark.parametrize("ctas", [1, 7])
@pytest.mark.parametrize("residency", ["miss", "partial"])
def test_launch_capped_to_few_ctas_matches_oracle(cuda, residency, ctas):
    """attend_ctas caps the IO/attention launch (SMs left to concurrent
    streams): one CTA, or seven, still fetch every block and attend every
    row, the plan's consumer count follows the cap, and outputs and read
    bytes are unchanged."""
    pool, cache, backing, source_q, source_pos, source_blocks, fetches = setup_case(residency)
    transport = GRSelectedTransport(cache, hot_policy="static", attend_ctas=ctas)
    try:
        for length in (13, 769):
            index = torch.arange(length, device="cuda") % len(source_q)
            query = source_q[index].contiguous()
            positions = source_pos[index].contiguous()
            blocks = source_blocks[index].contiguous()
            expected = _oracle(query, backing, blocks, positions)
            before = pool.read_bytes
            output, counters = transport.run(query, blocks, positions, fetches, 16)
            transport.last_done.synchronize()
            rows = counters.materialize()
            pool.flush_read_stats()
            torch.testing.assert_close(output.cpu().double(), expected, rtol=0.03, atol=0.03)
            assert pool.read_bytes - before == sum(r["misses"] for r in rows) * 256
            w = transport.workspace()
            assert w["consumer_ctas"] == min(w["rows"], 4 * ctas)
    finally:
        transport.close()
        pool.close()


@pytest.mark.parametrize("graphs", [False, True])
def test_poisoned_staging_hot_commit_and_graph(cuda, graphs):
    """tests/test_nsa_tma_transport.py:68-165 (poisoned KV / ready, exact hot commit)."""
    pool, cache, backing, query, positions, blocks, fetches = setup_case("partial")
    backing[73:] = torch.nan  # unrequested suffix values must never leak
    positions.clamp_max_(72)
    for head, fetch in enumerate(fetches):
        fetch["current_kv"].copy_(backing[67:, head])
    transport = GRSelectedTransport(cache, cuda_graphs=graphs)
    try:
        for state in ("partial", "miss", "hit", "empty"):
            query.mul_(-0.75)
            backing[67:73].add_(0.25)
            for head, fetch in enumerate(fetches):
                fetch["current_kv"].copy_(backing[67:, head])
            if state != "partial":
                cache.tags.fill_(-1)
            if state == "miss":
                blocks[:, 0] = torch.tensor([2, 4, 2, -1], device="cuda")
                blocks[:, 1] = torch.tensor([1, 0, 4, -1], device="cuda")
            elif state == "hit":
                for head in range(2):
                    cache.tags[head, :67] = torch.arange(67, device="cuda")
                    cache.data[cache.locs[head, :67].long()] = backing[:67, head].cuda()
            elif state == "empty":
                blocks.fill_(-1)
            blocks[3] = -1
            positions[7], blocks[7] = -1, -1
            hot = [set(row.tolist()) - {-1} for row in cache.tags.cpu()]
            needed = [set(), set()]
            for selected, position in zip(blocks.cpu().tolist(), positions.cpu().tolist()):
                for head, row in enumerate(selected):
                    for block in row:
                        if block >= 0:
                            needed[head].update(range(block * 16,
                                                      min(block * 16 + 16, position + 1, 67)))
            expected_bytes = sum(len(t - h) for t, h in zip(needed, hot)) * 256
            expected = _oracle(query, backing, blocks, positions)
            if transport.workspaces:
                w = transport.workspace()
                w["kv"].fill_(torch.nan)
                w["ready"].fill_(73)
            before = pool.read_bytes
            output, counters = transport.run(query, blocks, positions, fetches, 16)
            transport.last_done.synchronize()
            counters.materialize()
            pool.flush_read_stats()
            torch.testing.assert_close(output.cpu().double(), expected, rtol=0.03, atol=0.03)
            assert pool.read_bytes - before == expected_bytes
            w = transport.workspace()
            assert torch.all(w["ready"] == 1)
            for head in range(2):
                tags = cache.tags[head].cpu()
                occupied = tags >= 0
                assert set(tags[occupied].tolist()) == needed[head]
                locations = cache.locs[head].cpu()[occupied].long()
                actual = cache.data[locations.cuda()].cpu()
                assert torch.equal(actual.view(torch.uint8),
                                   backing[tags[occupied].long(), head].contiguous().view(torch.uint8))
        if graphs:
            assert transport.captures == 1 and transport.replays == 4
    finally:
        transport.close()
        pool.close()


@pytest.mark.parametrize("length,residency", [(128, "miss"), (256, "partial"), (769, "miss")])
def test_read_orders_preserve_output_plan_and_bytes(cuda, length, residency):
    pool, cache, backing, source_q, source_pos, source_blocks, fetches = setup_case(residency)
    index = torch.arange(length, device="cuda") % len(source_q)
    query = source_q[index].contiguous()
    positions = source_pos[index].contiguous()
    blocks = source_blocks[index].contiguous()
    blocks[: length // 2, 0] = torch.tensor([1, 0, 0, 4], device="cuda")
    positions[7] = -1
    blocks[7] = -1
    reference = None
    try:
        for order in ("physical", "consumption_depth", "consumption_depth_shared"):
            transport = GRSelectedTransport(cache, read_order=order, hot_policy="static",
                                            cuda_graphs=True)
            before = pool.read_bytes
            output, _ = transport.run(query, blocks, positions, fetches, 16)
            transport.last_done.synchronize()
            pool.flush_read_stats()
            w = transport.workspace()
            current = dict(output=output.cpu(), read_bytes=pool.read_bytes - before,
                           plan={k: w[k].cpu() for k in ("all_ids", "all_counts", "slots",
                                                         "valid", "flags")})
            assert torch.isfinite(current["output"]).all() and current["read_bytes"] > 0
            if reference is None:
                reference = current
            else:
                torch.testing.assert_close(current["output"], reference["output"],
                                           rtol=0.025, atol=0.004)
                assert current["read_bytes"] == reference["read_bytes"]
                for key, value in current["plan"].items():
                    assert torch.equal(value, reference["plan"][key]), key
            transport.close()
    finally:
        pool.close()


@pytest.mark.parametrize("residency", ["miss", "partial"])
def test_query_private_plan_reads_more_and_matches(cuda, residency):
    pool, cache, backing, query, positions, blocks, fetches = setup_case(residency)
    outputs, misses = [], []
    try:
        for dedup in (True, False):
            transport = GRSelectedTransport(cache, cross_query_dedup=dedup, hot_policy="static")
            output, counters = transport.run(query, blocks, positions, fetches, 16)
            transport.last_done.synchronize()
            outputs.append(output.cpu().double())
            misses.append(sum(r["misses"] for r in counters.materialize()))
            transport.close()
        expected = _oracle(query, backing, blocks, positions)
        for out in outputs:
            torch.testing.assert_close(out, expected, rtol=0.03, atol=0.03)
        assert misses[1] > misses[0]
    finally:
        pool.close()


def test_striped_regions_and_dram_backend(cuda):
    for backend, regions in (("host", 3), ("dram", 1)):
        pool, cache, backing, query, positions, blocks, fetches = setup_case(
            "miss", backend=backend, regions=regions)
        transport = GRSelectedTransport(cache, hot_policy="static")
        try:
            output, counters = transport.run(query, blocks, positions, fetches, 16)
            transport.last_done.synchronize()
            counters.materialize()
            expected = _oracle(query, backing, blocks, positions)
            torch.testing.assert_close(output.cpu().double(), expected, rtol=0.03, atol=0.03)
            w = transport.workspace()
            assert w["region_counts"].sum().item() == counters.statistics[:, 3].sum().item()
            if regions > 1:
                assert (w["region_counts"] > 0).sum().item() > 1
        finally:
            transport.close()
            pool.close()
