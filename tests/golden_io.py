"""Helpers to read the committed golden fixtures (tests/golden/*.npz)."""

from pathlib import Path

import numpy as np

GOLDEN = Path(__file__).resolve().parent / "golden"


def plan_fixtures():
    return sorted(GOLDEN.glob("plan_*.npz"))


def load(path):
    z = np.load(path)
    return {k: z[k] for k in z.files}


def oracle_args(z):
    return dict(
        blocks=z["blocks"], positions=z["positions"], desc=z["desc"], tags=z["tags"],
        locs=z["locs"], host_locs=z["host_locs"], hot_data=int(z["hot_data"]),
        bases=z["bases"], bs=int(z["bs"]), hot=int(z["hot"]),
        map_blocks=int(z["map_blocks"]), pool_tokens=int(z["pool_tokens"]),
        page_size=int(z["page_size"]), consumer_ctas=int(z["consumer_ctas"]),
        read_order=str(z["read_order"]))


EXACT_KEYS = ("active_counts", "required", "stats", "address", "hbm", "slots", "valid",
              "starts", "flags", "region_counts", "all_ids", "all_counts", "positions",
              "frequencies")
