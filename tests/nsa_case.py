"""Shared GPU fixture: a live host pool, hot cache and selections.

Restates the reference transport test geometry (tests/test_nsa_transport.py:97-144):
80 tokens x 2 KV heads, 67 cached history tokens in the backing pool, 13
suffix rows at positions 67..79, BS 16, duplicate block 0 and a shared causal
tail block 4 spanning history and suffix.
"""

import torch

from cxlsparse_b200.mempool import HiSparseCache, MemoryPool


def setup_case(residency, *, seed=71, hot=256, backend="host", regions=1):
    pool = MemoryPool(8, 128, backend, page_size=64, regions=regions)
    cache = HiSparseCache(pool, rows=2, max_history=256, hot=hot, topk=min(hot, 256), dim=128)
    g = torch.Generator().manual_seed(seed)
    backing = torch.randn(80, 2, 128, generator=g).bfloat16()
    query = torch.randn(13, 2, 16, 64, generator=g).bfloat16().cuda()
    positions = torch.arange(67, 80, device="cuda")
    blocks = torch.tensor([[[0, 1, 0, 4], [1, 0, 1, 4]]] * 13, dtype=torch.int32, device="cuda")
    if residency == "empty":
        blocks.fill_(-1)
    fetches = []
    for head in range(2):
        pages = pool.allocate(2)
        slots = pool.token_slots(pages, 0, 67)
        pool.write_many(slots, backing[:67, head].contiguous().cuda())
        cache.bind(head, slots)
        tokens = (list(range(67)) if residency == "hit"
                  else list(range(16)) + [17, 65] if residency == "partial" else [])
        tokens = tokens[:hot]
        if tokens:
            cache.tags[head, : len(tokens)] = torch.tensor(tokens, device="cuda", dtype=torch.int32)
            cache.data[cache.locs[head, : len(tokens)].long()] = backing[tokens, head].cuda()
        fetches.append(dict(row=head, cached_length=67, history_length=67,
                            current_kv=backing[67:, head].contiguous().cuda(), pages=pages))
    return pool, cache, backing, query, positions, blocks, fetches
