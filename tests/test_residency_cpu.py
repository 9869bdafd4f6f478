"""Residency table (HBM replica of any pattern) in the oracle planner, on CPU.

The reference decides residency with a hot hash of at most `hot` tokens per
cache row (planning/active.py:134-165). The table form (`hbm_locs[row,
token]`) must reproduce the hash plan exactly when it holds the same tokens,
and extends it to large or patterned replicas (recent blocks, blocks only
partly resident).
"""

import numpy as np
import pytest

from golden_io import load, oracle_args, plan_fixtures
from oracle import plan as P

KEYS = ("active_counts", "active_keys", "required", "stats", "address", "hbm", "slots",
        "valid", "starts", "flags", "region_counts", "all_ids", "all_counts", "ioids",
        "ranks", "frequencies")


def table_from_tags(args):
    """hbm_locs equivalent to the fixture's hot tags (first tag of a token wins)."""
    tags, locs, desc = args["tags"], args["locs"], args["desc"]
    rows, max_history = args["host_locs"].shape
    table = np.full((rows, max_history), -1, np.int64)
    for h in range(len(desc)):
        row, old = int(desc[h, 0]), int(desc[h, 1])
        for i in range(args["hot"]):
            t = int(tags[row, i])
            if 0 <= t < min(old, max_history) and table[row, t] < 0:
                table[row, t] = int(locs[row, i])
    return table


@pytest.mark.parametrize("path", plan_fixtures(), ids=lambda p: p.stem)
def test_table_equal_to_hot_tags_gives_the_reference_plan(path):
    z = load(path)
    args = oracle_args(z)
    planner = P.private_plan if int(z["private"]) else P.active_plan
    expected = planner(**args)
    got = planner(**args, hbm_locs=table_from_tags(args))
    for key in KEYS:
        assert np.array_equal(np.asarray(got[key]), np.asarray(expected[key])), key


def test_partly_resident_blocks_are_gathered():
    """A block with some tokens resident and some in the pool is a missing
    mixed-source block: kind 2 (token gather), its resident tokens from HBM."""
    z = load(plan_fixtures()[3])  # miss_bs64_shared_regions: every block cold
    args = oracle_args(z)
    rows, max_history = args["host_locs"].shape
    table = np.full((rows, max_history), -1, np.int64)
    bs = args["bs"]
    table[:, : bs // 2] = np.arange(bs // 2)  # first half of block 0 resident everywhere
    plan = P.active_plan(**args, hbm_locs=table)
    kinds, _ = P.source_kinds(plan["address"], plan["valid"], plan["flags"], bs)
    base = P.active_plan(**args)
    cap = plan["geometry"]["per_head"]
    for h in range(len(args["desc"])):
        keys = list(plan["active_keys"][h, : plan["active_counts"][h]])
        if 0 not in keys:
            continue
        p = h * cap + keys.index(0)
        req = int(plan["required"][h, keys.index(0)])
        assert plan["flags"][p] == 1 and kinds[p] == 2
        resident = min(req, bs // 2)
        assert plan["stats"][h, 2] == resident
        assert plan["stats"][h, 3] == base["stats"][h, 3] - resident
        for o in range(resident):
            assert plan["address"][p, o] == args["hot_data"] + o * 256
            assert plan["slots"][p * bs + o] == -1
