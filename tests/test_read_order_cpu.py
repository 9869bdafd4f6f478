"""The attention launch's CTA count only sets the planner's consumer count
(consumer c = row mod consumers, 4 attention warps per CTA). On every
reference planner fixture, the oracle plan at any consumer count fetches the
same blocks from the same sources; only the read order (IOIDs, ranks, first
depths) moves, and it stays a permutation of the missing blocks. That is
why a capped launch changes speed, never results."""

import numpy as np
import pytest

from golden_io import load, oracle_args, plan_fixtures
from oracle import plan as P

ORDER_KEYS = {"ioids", "ranks", "first_depth", "near", "consumer_ctas"}


@pytest.mark.parametrize("path", [p for p in plan_fixtures() if "private" not in p.stem],
                         ids=lambda p: p.stem)
def test_consumer_count_moves_only_the_read_order(path):
    z = load(path)
    args = oracle_args(z)
    rows = len(z["positions"]) * z["blocks"].shape[1]
    base = P.active_plan(**args)
    missing = int(base["missing"])
    wanted = np.flatnonzero(np.asarray(base["flags"])).tolist()
    moved = False
    for consumers in (1, 4, 7, 148, 592):
        args["consumer_ctas"] = max(1, min(rows, consumers))
        out = P.active_plan(**args)
        for key in base:
            if key in ORDER_KEYS or key == "geometry":
                continue
            assert np.array_equal(np.asarray(out[key]), np.asarray(base[key])), (consumers, key)
        assert int(out["missing"]) == missing
        order = np.asarray(out["ioids"])[:missing]
        assert sorted(order.tolist()) == wanted
        moved |= not np.array_equal(order, np.asarray(base["ioids"])[:missing])
    if str(z["read_order"]).startswith("consumption_depth") and missing:
        assert moved  # the depth orders do depend on the consumer count
