"""Device planner vs the oracle at the dedup stress size.

16 candidate queries x 128 extend tokens (2048 query rows) over an H=16384
history, 2 KV heads, top-16 blocks of 64 tokens, a hot replica of 256 tokens
per head, two pool regions. Selections overlap the way the dedup stress
workload's do (each 128-row candidate shares a base set of blocks, rows swap
some of them). Both the deduplicating plan and the query-private plan must
match the oracle bit-exactly at this size, and so must the fetched-byte
reduction computed from them.
"""

import numpy as np
import pytest
import torch

from golden_io import EXACT_KEYS
from oracle import plan as P
from test_gpu_planner import run_device_plan

pytestmark = pytest.mark.gpu

Q, H, W, BS, HISTORY, HOT = 2048, 2, 16, 64, 16384, 256


def _case(seed=7):
    rng = np.random.default_rng(seed)
    positions = (HISTORY + np.arange(Q)).astype(np.int32)
    blocks = np.empty((Q, H, W), np.int32)
    for start in range(0, Q, 128):
        for h in range(H):
            base = rng.choice(HISTORY // BS, W - 1, replace=False)
            for q in range(start, start + 128):
                current = positions[q] // BS
                row = base.copy()
                swap = rng.random(W - 1) < 0.3
                row[swap] = rng.integers(0, current, swap.sum())
                blocks[q, h] = np.concatenate(([current], row))
    blocks[5, 0, 3] = -1                      # a padded selection slot
    rows = H
    max_history = HISTORY + Q
    host_locs = np.full((rows, max_history), -1, np.int64)
    for r in range(rows):
        slots = r * HISTORY + np.arange(HISTORY)
        scramble = rng.choice(HISTORY // BS, 8, replace=False)  # a few non-contiguous blocks
        for b in scramble:
            seg = slots[b * BS:(b + 1) * BS]
            slots[b * BS:(b + 1) * BS] = seg[rng.permutation(BS)]
        host_locs[r, :HISTORY] = slots
    tags = np.full((rows, HOT + 1), -1, np.int32)
    locs = np.zeros((rows, HOT + 1), np.int32)
    for r in range(rows):
        tags[r, :HOT] = rng.choice(HISTORY, HOT, replace=False)
        locs[r, :] = r * (HOT + 1) + np.arange(HOT + 1)
    desc = np.array([(h, HISTORY, HISTORY, (1 << 40) + (h << 30), Q) for h in range(H)],
                    np.int64)
    map_blocks = max(64, -(-(HISTORY + Q) // (64 * BS)) * 64)
    return dict(blocks=blocks, positions=positions, desc=desc, tags=tags, locs=locs,
                host_locs=host_locs, hot_data=np.int64(1 << 42),
                bases=np.array([1 << 44, (1 << 44) + (1 << 36)], np.int64), bs=np.int64(BS),
                hot=np.int64(HOT), map_blocks=np.int64(map_blocks),
                pool_tokens=np.int64(H * HISTORY), page_size=np.int64(64),
                consumer_ctas=np.int64(592), read_order=np.array("consumption_depth"),
                private=np.int64(0))


def _oracle_args(z, private):
    return dict(blocks=z["blocks"], positions=z["positions"], desc=z["desc"], tags=z["tags"],
                locs=z["locs"], host_locs=z["host_locs"], hot_data=int(z["hot_data"]),
                bases=z["bases"], bs=BS, hot=HOT, map_blocks=int(z["map_blocks"]),
                pool_tokens=int(z["pool_tokens"]), page_size=64,
                consumer_ctas=None if private else 592,
                read_order="physical" if private else "consumption_depth")


def _compare(w, ref):
    cpu = {k: v.cpu().numpy() for k, v in w.items() if isinstance(v, torch.Tensor)}
    for key in EXACT_KEYS:
        assert np.array_equal(cpu[key].astype(np.int64).reshape(-1),
                              np.asarray(ref[key]).astype(np.int64).reshape(-1)), key
    missing = int(cpu["missing"][0])
    assert missing == int(ref["missing"])
    assert np.array_equal(cpu["ioids"][:missing], ref["ioids"][:missing])
    flags = cpu["flags"].astype(bool)
    assert np.array_equal(cpu["ranks"][flags], ref["ranks"][flags])
    assert np.array_equal(cpu["chosen"], ref["chosen"])
    return int(cpu["stats"][:, 3].sum())


def test_full_size_dedup_and_private_plans_match_oracle(cuda):
    z = _case()
    shared_ref = P.active_plan(**_oracle_args(z, False))
    shared = _compare(run_device_plan(z, cuda), shared_ref)
    zp = dict(z, private=np.int64(1), read_order=np.array("physical"))
    private_ref = P.private_plan(**_oracle_args(zp, True))
    private = _compare(run_device_plan(zp, cuda, consumer_ctas=min(Q * H, 256)), private_ref)
    assert shared < private
    reduction = 1 - shared / private
    assert reduction == 1 - int(shared_ref["stats"][:, 3].sum()) / int(
        private_ref["stats"][:, 3].sum())
    assert 0.5 < reduction < 1.0
