"""Known-answer vectors from the reference's own tests, against the oracle.

tests/test_nsa_active_plan.py:15-109 (reference_active_plan semantics) and
tests/test_nsa_dependency_order.py:35-83 (consumption-depth queues). The
reference describes sources as per-fetch dicts; the adapter below turns them
into the cache tensors (tags / locs / host_locs) the planner reads.
"""

import numpy as np
import pytest

from oracle import plan as P

HOT_DATA = 1 << 40
CURRENT = 1 << 44
BASE = 1 << 32


def _fetch(old=19, history=19, total=25, hot=(), offset=0):
    return dict(cached_length=old, history_length=history, total_length=total,
                hot_locations={t: offset + 100 + i for i, t in enumerate(hot)},
                host_slots={t: offset + t * 3 for t in range(old)})


def _run(blocks, positions, fetches, *, bs, hot):
    blocks = np.asarray(blocks, np.int64)
    heads = len(fetches)
    hot_cap = max(hot, 64)
    tags = np.full((heads, hot_cap + 1), -1, np.int64)
    locs = np.zeros((heads, hot_cap + 1), np.int64)
    max_history = 64
    host_locs = np.full((heads, max_history), -1, np.int64)
    desc = np.zeros((heads, 5), np.int64)
    for h, f in enumerate(fetches):
        for i, (t, loc) in enumerate(f["hot_locations"].items()):
            tags[h, i], locs[h, i] = t, loc
        for t, s in f["host_slots"].items():
            host_locs[h, t] = s
        desc[h] = (h, f["cached_length"], f["history_length"], CURRENT,
                   f["total_length"] - f["cached_length"])
    needed = max(f["total_length"] for f in fetches)
    plan = P.active_plan(blocks, positions, desc, tags, locs, host_locs, HOT_DATA, [BASE],
                         bs=bs, hot=hot_cap, map_blocks=-(-needed // bs), pool_tokens=1 << 20,
                         page_size=1 << 20, read_order="physical")
    return plan


def _sources(plan, head, block, bs):
    cap = plan["geometry"]["per_head"]
    keys = list(plan["active_keys"][head, : plan["active_counts"][head]])
    p = head * cap + keys.index(block)
    out = []
    for o in range(int(plan["required"][head, keys.index(block)])):
        a = int(plan["address"][p, o])
        if plan["slots"][p * bs + o] >= 0:
            out.append(("external", int(plan["slots"][p * bs + o])))
        elif a >= CURRENT:
            out.append(("current", (a - CURRENT) // 256))
        else:
            out.append(("hot", (a - HOT_DATA) // 256))
    return tuple(out)


def _hot_tokens(plan, head, bs, hot):
    keys = plan["active_keys"][head]
    out = []
    for ct in plan["chosen"][head, :hot]:
        if plan["frequencies"][head, ct] > 0:
            out.append(int(keys[ct // bs]) * bs + int(ct % bs))
    return tuple(out)


def test_duplicate_occurrences_partial_hits_and_causal_tail():
    plan = _run([[[0, 0, 2]], [[0, 1, 2]]], [19, 24], [_fetch(hot=(0, 2, 16, 18))], bs=8, hot=32)
    assert list(plan["active_keys"][0, :3]) == [0, 1, 2]
    assert list(plan["required"][0, :3]) == [8, 8, 8]
    assert plan["all_ids"][0, :3].tolist() == [0, 0, 2]
    assert _sources(plan, 0, 0, 8)[0] == ("hot", 100)
    assert _sources(plan, 0, 0, 8)[1] == ("external", 3)
    assert _sources(plan, 0, 2, 8)[:4] == (("hot", 102), ("external", 51), ("hot", 103),
                                           ("current", 0))
    assert _hot_tokens(plan, 0, 8, 32) == tuple(range(8)) + (16, 17, 18) + tuple(range(8, 16))
    assert tuple(plan["stats"][0]) == (24, 19, 4, 15, 38, 6, 0)


@pytest.mark.parametrize("mode", ["miss", "hit", "empty"])
def test_empty_and_full_residency(mode):
    blocks = np.array([[[0, 1]], [[0, 2]]])
    if mode == "empty":
        blocks[:] = -1
    plan = _run(blocks, [19, 24], [_fetch(hot=range(19) if mode == "hit" else ())], bs=8, hot=7)
    assert plan["stats"][0][3] == (19 if mode == "miss" else 0)
    assert plan["stats"][0][2] == (19 if mode == "hit" else 0)
    if mode == "empty":
        assert plan["active_counts"][0] == 0 and tuple(plan["stats"][0]) == (0,) * 7
    else:
        assert _hot_tokens(plan, 0, 8, 7) == tuple(range(7))


def test_padded_rows_do_not_select():
    blocks = [[[1, 1]], [[-1, -1]], [[0, 2]]]
    padded = _run(blocks, [19, -1, -1], [_fetch()], bs=8, hot=32)
    alone = _run(blocks[:1], [19], [_fetch()], bs=8, hot=32)
    assert np.array_equal(padded["stats"], alone["stats"])
    assert padded["all_counts"].tolist() == [2, 0, 0]


def test_owner_heads_and_backing_replacement():
    plan = _run([[[2], [2]]], [24], [_fetch(hot=(16,)), _fetch(offset=1000)], bs=8, hot=32)
    assert _sources(plan, 0, 2, 8)[0] == ("hot", 100)
    assert _sources(plan, 1, 2, 8)[0] == ("external", 1048)
    replay = _run([[[2]]], [24], [_fetch(old=23, history=23, total=29, hot=(21,), offset=2000)],
                  bs=8, hot=32)
    s = _sources(replay, 0, 2, 8)
    assert s[0] == ("external", 2048) and s[5] == ("hot", 2100) and s[7] == ("current", 0)
    assert _hot_tokens(replay, 0, 8, 32) == tuple(range(16, 23))


def test_invalid_selection_counts_errors():
    plan = _run([[[4]]], [24], [_fetch()], bs=8, hot=8)
    assert plan["stats"][0][6] == 1
    assert plan["all_counts"].tolist() == [0]


def _dep_case():
    return dict(ids=np.array([[2, 2, 2, 3, 2, 2], [3, 0, 0, 0, 2, 5], [1, 4, -1, -1, -1, -1],
                              [1, 1, 1, 1, -1, -1], [7, 7, 7, 7, 7, 7], [4, -1, -1, -1, -1, -1]]),
                counts=np.array([6, 6, 2, 4, 0, 1]), flags=np.array([0, 1, 1, 1, 1, 1, 1, 1]),
                positions=np.array([7, 7, 8, 8, -1, 9]))


def test_dependency_queue_resident_steps_and_near_ties():
    c = _dep_case()
    ioids, _, missing, first, near, _ = P.consumption_order(
        c["ids"], c["counts"], c["positions"], c["flags"], 2, 6)
    assert ioids[:missing].tolist() == [2, 3, 5, 1, 4, 6, 7]
    assert [first[b] for b in (2, 3, 5, 1, 4)] == [0, 0, 5, 6, 7]
    ioids, _, missing, first, near, _ = P.consumption_order(
        c["ids"], c["counts"], c["positions"], c["flags"], 2, 6, shared=True)
    assert ioids[:missing].tolist() == [3, 2, 5, 1, 4, 6, 7]
    assert near[2] == 1 and near[3] == 2 and near[4] == 2 and near[6] == near[7] == 0


def test_dependency_distinct_rows_reusing_one_consumer():
    ioids, _, missing, first, near, _ = P.consumption_order(
        np.array([[2, 1], [1, 0], [2, -1], [-1, -1], [2, -1]]), np.array([2, 2, 1, 0, 1]),
        np.array([0, 0, 1, -1, 2]), np.array([0, 1, 1]), 2, 2, shared=True)
    assert first[1] == 0 and first[2] == 0
    assert near[1] == 2 and near[2] == 3
    assert ioids[:missing].tolist() == [2, 1]


@pytest.mark.parametrize("error_head", [-1, 0, 1])
def test_occurrence_rows_keep_duplicates_order_and_exclude_invalid_rows(error_head):
    """tests/test_nsa_tma_plan.py:43-96: occurrence rows from a given mapping.
    Duplicates stay in selection order; blocks out of range, in the causal
    future, unmapped (-1 / -2) or mapped past the per-head capacity drop out;
    padded rows and every row of a head with an error count are empty."""
    blocks = np.array([
        [[1, 0, 0, 2, -1, 6, 3], [1, 0, 1, -1, 2, 6, 0]],
        [[4, 2, 2, 3, 0, 5, -1], [4, 3, 2, 1, 0, -1, 6]],
        [[0, 0, 1, 2, 3, 4, 5], [1, 2, 3, 4, 5, 0, 0]],
    ])
    positions = np.array([31, 79, -1])
    mapping = np.array([[2, -1, 0, 4, -2, 3, -2], [1, 0, 3, 2, 4, -1, -2]])
    errors = np.zeros(2, np.int64)
    if error_head >= 0:
        errors[error_head] = 1
    ids, counts, rows_pos = P.occurrence_rows(
        blocks, positions, lambda h, b: mapping[h, b], errors, bs=16, map_blocks=6, per_head=4)
    # Query 0 (pos 31) sees blocks 0-1, query 1 (pos 79) blocks 0-4.
    head0_q0 = [4 * 0 + 2, 4 * 0 + 2]            # blocks 1 (-1: dropped), 0, 0
    head1_q0 = [4 + 0, 4 + 1, 4 + 0, 4 + 1]       # blocks 1, 0, 1, 0 -> compact 0, 1, 0, 1
    head0_q1 = [4 * 0 + 0, 4 * 0 + 0, 0 + 2]      # 4 -> -2, 2, 2, 3 -> 4 (>= cap), 0 -> 2
    head1_q1 = [4 + 2, 4 + 3, 4 + 0, 4 + 1]       # 4 -> 4 (>= cap), 3, 2, 1, 0
    expected = {0: head0_q0, 1: head1_q0, 2: head0_q1, 3: head1_q1, 4: [], 5: []}
    for row, want in expected.items():
        if error_head >= 0 and row % 2 == error_head:
            want = []
        assert counts[row] == len(want), row
        assert list(ids[row, : len(want)]) == want, row
        assert (ids[row, len(want):] == -1).all()
    assert list(rows_pos) == [31, 31, 79, 79, -1, -1]


def test_prepare_classification_table():
    """tests/test_nsa_tma_prepare.py:7-105: the seven source classes of a
    physical block. Only a missing block of BS contiguous, 16-byte aligned
    external tokens is a bulk copy (kind 1, its first address as source);
    other missing blocks are token gathers (kind 2); resident and inactive
    blocks are kind 0 and ready from the start."""
    bs, external, resident = 16, 1 << 20, 9 << 20
    cases = ["inactive", "direct", "resident", "mixed", "tail", "hot_tail", "gather"]
    address = np.zeros((len(cases), bs), np.int64)
    valid = np.zeros(len(cases), np.int64)
    flags = np.zeros(len(cases), np.int64)
    for p, kind in enumerate(cases):
        count = {"inactive": 0, "tail": 5, "hot_tail": 7}.get(kind, bs)
        valid[p] = count
        flags[p] = kind in ("direct", "mixed", "tail", "gather")
        t = np.arange(bs)
        if kind == "direct":
            address[p] = external + t * 256
        elif kind in ("resident", "hot_tail"):
            address[p, :count] = resident + t[:count] * 256
        elif kind == "mixed":
            address[p] = np.where(t % 2 == 0, external + t * 256, resident + t * 256)
        elif kind == "tail":
            address[p, :count] = external + (16 + t[:count]) * 256
        elif kind == "gather":
            address[p] = external + (bs - 1 - t) * 256
    kinds, first = P.source_kinds(address, valid, flags, bs)
    assert list(kinds) == [0, 1, 0, 2, 2, 0, 2]
    assert first[1] == external
    assert list(1 - flags) == [1, 0, 1, 0, 0, 1, 0]  # ready from the start
