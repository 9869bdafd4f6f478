"""Candidate segments on the CPU: the layout helper, and the oracle planner run
in segment positions.

Several GR candidates share one history; each must see the history and its
own suffix only. The path expresses that purely through positions (see
``cxlsparse_b200/segments.py``), so the planner is the unchanged
deduplicating plan of planning/active.py. These tests run the numpy oracle of
that plan on segment positions and check, token by token, that every row
reads exactly the sources its candidate would read on its own: pool slots
for shared history, its own current KV for the history tail and its suffix,
with history blocks fetched once for all candidates.
"""

import random

import numpy as np
import pytest

from cxlsparse_b200.segments import SegmentLayout
from oracle import plan as P

BASE = 1 << 32
CURRENT = 1 << 44


@pytest.mark.parametrize("seed", range(20))
def test_layout_round_trips(seed):
    rng = random.Random(seed)
    bs = rng.choice([16, 32, 64])
    layout = SegmentLayout(rng.randrange(0, 5000), rng.randrange(1, 300), rng.randrange(1, 9), bs)
    assert layout.start % bs == 0 and layout.tokens % bs == 0
    assert layout.start + layout.tail == layout.history
    assert layout.tokens >= layout.tail + layout.extend
    assert layout.tokens == -(-(layout.extend + bs - 1) // bs) * bs  # same for every tail
    positions = layout.positions()
    assert len(positions) == layout.candidates * layout.extend
    for row, pos in enumerate(positions):
        c, i = divmod(row, layout.extend)
        assert layout.true_position(pos) == layout.history + i
        assert layout.candidate_of(pos) == c
        block = layout.true_position(pos) // bs
        assert layout.segment_block(c, block) == pos // bs
        assert layout.true_block(pos // bs) == block
    # Segments of different candidates never share a block.
    owners = {}
    for row, pos in enumerate(positions):
        c = row // layout.extend
        assert owners.setdefault(pos // bs, c) == c
    for t in range(layout.start):
        assert layout.true_position(t) == t and layout.candidate_of(t) is None


def _plan(history, extend, candidates, bs, width, seed, heads=2):
    """Random true-coordinate selections per candidate row, mapped to segment
    blocks and planned by the oracle (no hot replica: every history token is
    a pool slot)."""
    layout = SegmentLayout(history, extend, candidates, bs)
    rng = np.random.default_rng(seed)
    rows = candidates * extend
    positions = np.array(layout.positions(), np.int64)
    blocks = np.full((rows, heads, width), -1, np.int64)
    true_sel = {}
    for row in range(rows):
        c, i = divmod(row, extend)
        true_pos = history + i
        current = true_pos // bs
        for h in range(heads):
            earlier = rng.permutation(current)[: width - 1] if current else []
            chosen = [current] + [int(b) for b in earlier]
            # Duplicates are legal occurrences and must be attended again.
            if len(chosen) < width and rng.random() < 0.3:
                chosen.append(chosen[-1])
            true_sel[row, h] = chosen
            blocks[row, h, : len(chosen)] = [layout.segment_block(c, b) for b in chosen]
    host_locs = np.full((heads, layout.start + layout.tokens), -1, np.int64)
    slot_of = {}
    for h in range(heads):
        for t in range(history):  # pool slots of the whole true history
            slot_of[h, t] = 7 * t + 3 * h
            host_locs[h, t] = slot_of[h, t]
    desc = np.array([(h, layout.start, layout.start, CURRENT + h * (1 << 36),
                      candidates * layout.tokens) for h in range(heads)], np.int64)
    tags = np.full((heads, 65), -1, np.int64)
    locs = np.zeros((heads, 65), np.int64)
    needed = layout.start + candidates * layout.tokens
    plan = P.active_plan(blocks, positions, desc, tags, locs, host_locs, 1 << 40, [BASE],
                         bs=bs, hot=64, map_blocks=-(-needed // bs), pool_tokens=1 << 30,
                         page_size=1 << 30, read_order="consumption_depth")
    return layout, positions, true_sel, slot_of, desc, plan


@pytest.mark.parametrize("history,extend,candidates,bs", [
    (150, 20, 3, 16),    # history tail of 6 tokens carried into each segment
    (128, 16, 4, 16),    # block-aligned history: no tail
    (1000, 64, 5, 64),   # tail 40 + 64 suffix tokens: two blocks per segment
    (70, 100, 2, 32),    # suffix longer than the history
])
def test_oracle_plan_reads_each_candidates_own_tokens(history, extend, candidates, bs):
    width, heads = 6, 2
    layout, positions, true_sel, slot_of, desc, plan = _plan(
        history, extend, candidates, bs, width, seed=history + candidates, heads=heads)
    assert not plan["stats"][:, 6].any()
    cap = plan["geometry"]["per_head"]
    for row in range(candidates * extend):
        c, i = divmod(row, extend)
        true_pos = history + i
        for h in range(heads):
            r = row * heads + h
            ids = plan["all_ids"][r, : plan["all_counts"][r]]
            assert len(ids) == len(true_sel[row, h])
            seen_blocks = []
            for p, true_block in zip(ids, true_sel[row, h]):
                start = int(plan["starts"][p])
                assert layout.true_block(start // bs) == true_block
                assert p // cap == h
                seen_blocks.append(true_block)
                for o in range(bs):
                    seg_pos = start + o
                    if seg_pos > positions[row]:
                        break  # beyond the row: masked by the attention kernel
                    t = layout.true_position(seg_pos)
                    assert t <= true_pos
                    address = int(plan["address"][p, o])
                    if t < layout.start:
                        assert address == BASE + slot_of[h, t] * 256
                    else:  # history tail or own suffix: the candidate's segment
                        assert address == int(desc[h, 3]) + (c * layout.tokens + t - layout.start) * 256
            assert seen_blocks == true_sel[row, h]
    # History blocks are planned once per head whichever candidates chose them.
    first = layout.start // bs
    for h in range(heads):
        keys = [int(k) for k in plan["active_keys"][h, : plan["active_counts"][h]]]
        history_keys = [k for k in keys if k < first]
        chosen = {b for (row, hh), sel in true_sel.items() if hh == h for b in sel if b < first}
        assert sorted(history_keys) == sorted(chosen)
        # Suffix blocks: one per (candidate, block) that candidate selected.
        private = {(row // extend, b) for (row, hh), sel in true_sel.items() if hh == h
                   for b in sel if b >= first}
        assert len(keys) - len(history_keys) == len(private)


def test_segments_fetch_history_once():
    """Misses of the segment plan = unique history tokens selected by any
    candidate (the suffix is current KV): what the deduplicating plan saves
    over planning each candidate on its own."""
    history, extend, candidates, bs = 1000, 64, 5, 64
    layout, positions, true_sel, slot_of, desc, plan = _plan(history, extend, candidates, bs,
                                                             6, seed=3)
    first = layout.start // bs
    for h in range(2):
        blocks = {b for (row, hh), sel in true_sel.items() if hh == h for b in sel if b < first}
        per_candidate = sum(
            len({b for (row, hh), sel in true_sel.items()
                 if hh == h and row // extend == c for b in sel if b < first})
            for c in range(candidates))
        assert plan["stats"][h, 3] == len(blocks) * bs
        assert per_candidate > len(blocks)
