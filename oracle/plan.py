"""Numpy restatement of the deduplicating selected-block planner (test oracle).

Follows ``cxl_recsys/models/nsa/planning/active.py`` (``ActivePlanAdapter``),
``planning/occurrences.py``, ``planning/dependencies.py`` and
``tma/transport.py:_prepare_sources``. Every output array has the meaning and
layout of the reference workspace entry of the same name, so a device plan can
be compared element by element.

Inputs use the reference's descriptor convention: ``desc`` is [H, 5] int64 of
(cache row, cached_length, history_length, current_kv address, current length)
(``models/nsa/transport.py:585-604``).
"""

import math

import numpy as np

INT32_MAX = 2147483647
TOKEN_BYTES = 256  # one KV token = 64 K + 64 V bf16 (models/nsa/config.py:76-79)


def next_pow2(x):
    return 1 << max(0, int(x) - 1).bit_length()


def geometry(queries, heads, width, bs, hot, *, map_blocks, needed_tokens,
             private=False):
    """Capacity geometry (planning/active.py:517-552; query_private.py:222-241)."""
    if bs < 1 or bs & (bs - 1) or not heads or not width or not queries:
        raise ValueError("Nonempty geometry and a power-of-two block size required")
    needed = math.ceil(needed_tokens / bs)
    if map_blocks is None:
        map_blocks = needed
    if map_blocks < needed or map_blocks < 1:
        raise ValueError("History mapping capacity cannot truncate a request")
    if map_blocks * bs > INT32_MAX:
        raise ValueError("Absolute token addressing must fit int32")
    if private:
        per_head = queries * width
        sort_extent = max(map_blocks * bs, hot)
    else:
        per_head = min(map_blocks, queries * width)
        sort_extent = max(per_head * bs, hot)
    return dict(
        heads=heads, width=width, bs=bs, queries=queries, rows=queries * heads,
        map_blocks=map_blocks, per_head=per_head, physical=heads * per_head,
        sort_extent=sort_extent, hash_capacity=next_pow2(2 * hot), hot=hot,
    )


def _valid_occurrence(block, position, total, map_blocks, bs):
    """Per-slot selection validity (active.py:70-74, 98-102)."""
    return (position >= 0 and 0 <= block < map_blocks and block * bs <= position
            and block * bs < total)


def _hot_lookup(tags, locs, row, old, hot):
    """Token -> hot location for the owner row (active.py:134-165)."""
    table = {}
    for i in range(hot):
        token = int(tags[row, i])
        if 0 <= token < old and token not in table:
            table[token] = int(locs[row, i])
    return table


def _resolve(geo, keys_by_head, counts, required, desc, tags, locs, host_locs,
             hot_data, bases, pool_tokens, page_size, stats, region_counts, hbm_locs=None):
    """Per-token source resolution (active.py:209-295).

    ``hbm_locs`` [rows, max_history] (optional, not in the reference) replaces
    the hot tags: history token t of row r is resident at hot_data +
    hbm_locs[r, t] * 256 when that entry is >= 0."""
    heads, cap, bs, hot = geo["heads"], geo["per_head"], geo["bs"], geo["hot"]
    p_total = heads * cap
    address = np.zeros((p_total, bs), np.int64)
    hbm = np.zeros((p_total, bs), np.int64)
    slots = np.full((p_total, bs), -1, np.int64)
    valid = np.zeros(p_total, np.int32)
    starts = np.zeros(p_total, np.int32)
    flags = np.zeros(p_total, np.int32)
    regions = len(bases)
    max_history = host_locs.shape[1]
    for h in range(heads):
        row, old = int(desc[h, 0]), int(desc[h, 1])
        pointer = int(desc[h, 3])
        if hbm_locs is None:
            table = _hot_lookup(tags, locs, row, old, hot)
        else:
            table = {t: int(hbm_locs[row, t]) for t in range(min(old, hbm_locs.shape[1]))
                     if hbm_locs[row, t] >= 0}
        for c in range(cap):
            p = h * cap + c
            active = c < counts[h]
            if not active:
                continue
            block = int(keys_by_head[h][c])
            req = int(required[h, c])
            errors = 0
            any_external = False
            for o in range(bs):
                token = block * bs + o
                if o >= req:
                    continue
                stats[h, 0] += 1
                if token >= old:
                    hbm[p, o] = address[p, o] = pointer + (token - old) * TOKEN_BYTES
                    continue
                stats[h, 1] += 1
                location = table.get(token, -1)
                if location >= 0:
                    stats[h, 2] += 1
                    hbm[p, o] = address[p, o] = hot_data + location * TOKEN_BYTES
                    continue
                stats[h, 3] += 1
                any_external = True
                source = (int(host_locs[row, token])
                          if 0 <= token < max_history else -1)
                if source < 0 or source >= pool_tokens:
                    errors += 1
                    continue
                page = source // page_size
                region = page % regions
                local = (page // regions) * page_size + source % page_size
                address[p, o] = int(bases[region]) + local * TOKEN_BYTES
                slots[p, o] = source
                region_counts[region] += 1
            stats[h, 6] += errors
            valid[p] = req if errors == 0 else 0
            starts[p] = block * bs
            flags[p] = int(any_external)
    return address, hbm, slots, valid, starts, flags


def occurrence_rows(blocks, positions, compact_of, errors, *, bs, map_blocks, per_head):
    """Occurrence rows (planning/occurrences.py:7-55): row r = q * H + h lists,
    in the original selection order and with duplicates kept, head * per_head
    + compact for every block that is in range (0 <= b < map_blocks), causal
    (b * bs <= pos) and mapped to a compact slot in [0, per_head)
    (``compact_of(h, b)``). Padded rows (pos < 0) and every row of a head with
    a nonzero error count are empty. Returns (all_ids, all_counts, positions
    repeated per head)."""
    blocks = np.asarray(blocks, np.int64)
    q_count, heads, width = blocks.shape
    rows = q_count * heads
    all_ids = np.full((rows, width), -1, np.int32)
    all_counts = np.zeros(rows, np.int32)
    row_positions = np.zeros(rows, np.int64)
    for q in range(q_count):
        pos = int(positions[q])
        for h in range(heads):
            r = q * heads + h
            row_positions[r] = pos
            if errors[h] or pos < 0:
                continue
            n_valid = 0
            for i in range(width):
                b = int(blocks[q, h, i])
                if not (0 <= b < map_blocks and b * bs <= pos):
                    continue
                compact = int(compact_of(h, b))
                if 0 <= compact < per_head:
                    all_ids[r, n_valid] = h * per_head + compact
                    n_valid += 1
            all_counts[r] = n_valid
    return all_ids, all_counts, row_positions


def consumption_order(all_ids, all_counts, row_positions, flags, consumer_ctas,
                      width, *, shared=False, near_window=4):
    """Consumption-depth read order (planning/dependencies.py:37-300).

    Returns (ioids, ranks, missing, first, near, depth). Unreferenced missing
    blocks carry the sentinel depth cdiv(rows, consumers) * width and sort last.
    """
    rows = len(all_counts)
    n = len(flags)
    consumers = consumer_ctas
    max_depth = -(-rows // consumers) * width
    depth = np.zeros(rows, np.int32)
    first = np.full(n, max_depth, np.int64)
    for r in range(rows):
        d = 0
        for prev in range(r % consumers, r, consumers):
            if row_positions[prev] >= 0:
                d += int(all_counts[prev])
        depth[r] = d
        if row_positions[r] < 0:
            continue
        for col in range(min(width, int(all_counts[r]))):
            b = int(all_ids[r, col])
            if 0 <= b < n and flags[b]:
                first[b] = min(first[b], d + col)
    near = np.zeros(n, np.int32)
    if shared:
        for r in range(rows):
            if row_positions[r] < 0:
                continue
            seen = set()
            for col in range(min(width, int(all_counts[r]))):
                b = int(all_ids[r, col])
                if not (0 <= b < n and flags[b]):
                    continue
                d = int(depth[r]) + col
                if first[b] <= d < first[b] + near_window and b not in seen:
                    seen.add(b)
                    near[b] += 1
    missing_blocks = [b for b in range(n) if flags[b]]
    missing_blocks.sort(key=lambda b: (int(first[b]),
                                       -int(near[b]) if shared else 0, b))
    ioids = np.full(n, -1, np.int32)
    ranks = np.full(n, -1, np.int32)
    for rank, b in enumerate(missing_blocks):
        ioids[rank] = b
        ranks[b] = rank
    return ioids, ranks, len(missing_blocks), first, near, depth


def physical_order(flags):
    """Missing blocks in ascending physical order (active.py:298-305)."""
    n = len(flags)
    ioids = np.full(n, -1, np.int32)
    ranks = np.full(n, -1, np.int32)
    rank = 0
    for b in range(n):
        if flags[b]:
            ioids[rank] = b
            ranks[b] = rank
            rank += 1
    return ioids, ranks, rank


def hot_choice(frequencies, hot):
    """Top-`hot` indices by (frequency desc, index asc) (active.py:449-500, 863-888)."""
    heads = frequencies.shape[0]
    chosen = np.zeros((heads, hot), np.int64)
    for h in range(heads):
        order = np.argsort(-frequencies[h].astype(np.int64), kind="stable")
        chosen[h] = order[:hot]
    return chosen


def active_plan(blocks, positions, desc, tags, locs, host_locs, hot_data, bases,
                *, bs, hot, map_blocks, pool_tokens, page_size, consumer_ctas=None,
                read_order="consumption_depth", hbm_locs=None):
    """Full deduplicating plan; returns a dict of reference-workspace arrays.

    ``blocks`` [Q, H, W] int32, ``positions`` [Q] (negative = padded row).
    Cross-row duplicates of (head, block) share one compact slot; every row
    keeps its own occurrences, multiplicity and causal mask.
    """
    blocks = np.asarray(blocks, np.int64)
    positions = np.asarray(positions, np.int64)
    desc = np.asarray(desc, np.int64)
    q_count, heads, width = blocks.shape
    needed = max(int(desc[h, 1] + desc[h, 4]) for h in range(heads))
    geo = geometry(q_count, heads, width, bs, hot, map_blocks=map_blocks,
                   needed_tokens=needed)
    cap, mb = geo["per_head"], geo["map_blocks"]
    stats = np.zeros((heads, 7), np.int64)
    # Insert / dedup (active.py:56-114): first-seen order is irrelevant because
    # compact indices are the ranks of the sorted active keys (active.py:744-756).
    unique = [set() for _ in range(heads)]
    for q in range(q_count):
        pos = int(positions[q])
        for h in range(heads):
            total = int(desc[h, 1] + desc[h, 4])
            for i in range(width):
                b = int(blocks[q, h, i])
                if _valid_occurrence(b, pos, total, mb, bs):
                    unique[h].add(b)
                elif b >= 0 and pos >= 0:
                    stats[h, 6] += 1
    keys = []
    counts = np.zeros(heads, np.int32)
    active_keys = np.full((heads, cap), INT32_MAX, np.int64)
    for h in range(heads):
        ordered = sorted(unique[h])
        if len(ordered) > cap:
            stats[h, 6] += len(ordered) - cap
            ordered = ordered[:cap]  # which keys survive is unspecified on overflow
        keys.append(ordered)
        counts[h] = len(ordered)
        active_keys[h, : len(ordered)] = ordered
    mapping = [{b: c for c, b in enumerate(k)} for k in keys]
    # References (active.py:168-206).
    required = np.zeros((heads, cap), np.int64)
    frequencies = np.zeros((heads, geo["sort_extent"]), np.int64)
    for q in range(q_count):
        pos = int(positions[q])
        for h in range(heads):
            old, history = int(desc[h, 1]), int(desc[h, 2])
            total = old + int(desc[h, 4])
            for i in range(width):
                b = int(blocks[q, h, i])
                if not _valid_occurrence(b, pos, total, mb, bs) or b not in mapping[h]:
                    continue
                c = mapping[h][b]
                required[h, c] = max(required[h, c], min(bs, min(pos + 1, total) - b * bs))
                for o in range(bs):
                    t = b * bs + o
                    if t <= pos and t < total:
                        if t < history:
                            frequencies[h, c * bs + o] += 1
                        stats[h, 4 if t < old else 5] += 1
    region_counts = np.zeros(len(bases), np.int64)
    address, hbm, slots, valid, starts, flags = _resolve(
        geo, keys, counts, required, desc, tags, locs, host_locs, hot_data, bases,
        pool_tokens, page_size, stats, region_counts, hbm_locs)
    # Occurrence rows (occurrences.py:7-35): original order, duplicates kept.
    rows = q_count * heads
    all_ids, all_counts, row_positions = occurrence_rows(
        blocks, positions, lambda h, b: mapping[h].get(b, -1), stats[:, 6], bs=bs,
        map_blocks=mb, per_head=cap)
    if consumer_ctas is None:
        consumer_ctas = min(rows, 256)
    if read_order == "physical":
        ioids, ranks, missing = physical_order(flags)
        first = near = None
    else:
        ioids, ranks, missing, first, near, _ = consumption_order(
            all_ids, all_counts, row_positions, flags, consumer_ctas, width,
            shared=read_order == "consumption_depth_shared")
    chosen = hot_choice(frequencies, hot)
    return dict(
        geometry=geo, active_counts=counts, active_keys=active_keys,
        required=required, stats=stats, address=address, hbm=hbm,
        slots=slots.reshape(-1), valid=valid, starts=starts, flags=flags,
        region_counts=region_counts, all_ids=all_ids, all_counts=all_counts,
        positions=row_positions, ioids=ioids, ranks=ranks, missing=missing,
        first_depth=first, near=near, frequencies=frequencies, chosen=chosen,
        consumer_ctas=consumer_ctas,
    )


def source_kinds(address, valid, flags, bs):
    """Block source class (tma/transport.py:17-42), generalised to any BS.

    0 resident, 1 full contiguous 16-byte aligned external block (bulk copy),
    2 mixed-tier or tail block (token gather). Returns (kinds, first address).
    """
    p_total = len(valid)
    kinds = np.zeros(p_total, np.int32)
    first = address[:, 0].copy()
    for p in range(p_total):
        if not flags[p]:
            continue
        contiguous = all(int(address[p, t]) == int(first[p]) + t * TOKEN_BYTES
                         for t in range(bs))
        full = (valid[p] == bs and first[p] != 0 and first[p] % 16 == 0
                and contiguous)
        kinds[p] = 1 if full else 2
    return kinds, first


def retain_hot(plan, desc, tags, locs, *, bs, hot):
    """Hot commit of the chosen compact tokens (active.py:410-437, 909-925).

    Returns new tags and a list of (location, head, compact_token) payload moves.
    """
    tags = tags.copy()
    cap = plan["geometry"]["per_head"]
    moves = []
    for h in range(plan["geometry"]["heads"]):
        row = int(desc[h, 0])
        for slot in range(hot):
            ct = int(plan["chosen"][h, slot])
            selected = plan["frequencies"][h, ct] > 0
            compact = ct // bs
            if selected and compact < cap:
                token = int(plan["active_keys"][h, compact]) * bs + ct % bs
                tags[row, slot] = token
                moves.append((int(locs[row, slot]), h, ct))
            else:
                tags[row, slot] = -1
    return tags, moves


def private_plan(blocks, positions, desc, tags, locs, host_locs, hot_data, bases,
                 *, bs, hot, map_blocks, pool_tokens, page_size,
                 consumer_ctas=None, read_order="consumption_depth", hbm_locs=None):
    """Query-private (no cross-row sharing) plan (planning/query_private.py:29-457).

    Each (row query, head, block) owns a payload slot; repeats inside one query
    share that query's slot. Frequencies and the hot choice use absolute tokens
    and a canonical (lowest) private source per token for the hot commit.
    """
    blocks = np.asarray(blocks, np.int64)
    positions = np.asarray(positions, np.int64)
    desc = np.asarray(desc, np.int64)
    q_count, heads, width = blocks.shape
    needed = max(int(desc[h, 1] + desc[h, 4]) for h in range(heads))
    geo = geometry(q_count, heads, width, bs, hot, map_blocks=map_blocks,
                   needed_tokens=needed, private=True)
    cap, mb = geo["per_head"], geo["map_blocks"]
    stats = np.zeros((heads, 7), np.int64)
    private_keys = np.full((heads, cap), INT32_MAX, np.int64)
    private_required = np.zeros((heads, cap), np.int64)
    occurrences = np.full((q_count, heads, width), -1, np.int64)
    frequencies = np.zeros((heads, geo["sort_extent"]), np.int64)
    canonical = np.full((heads, geo["sort_extent"]), INT32_MAX, np.int64)
    for q in range(q_count):
        pos = int(positions[q])
        for h in range(heads):
            old, history = int(desc[h, 1]), int(desc[h, 2])
            total = old + int(desc[h, 4])
            row_blocks = [int(b) for b in blocks[q, h]]
            valid = [_valid_occurrence(b, pos, total, mb, bs) for b in row_blocks]
            own = sorted({b for b, v in zip(row_blocks, valid) if v})
            for i, b in enumerate(own):
                private_keys[h, q * width + i] = b
                private_required[h, q * width + i] = min(bs, min(pos + 1, total) - b * bs)
            for i, (b, v) in enumerate(zip(row_blocks, valid)):
                if not v:
                    if b >= 0 and pos >= 0:
                        stats[h, 6] += 1
                    continue
                origin = q * width + own.index(b)
                occurrences[q, h, i] = origin
                for o in range(bs):
                    t = b * bs + o
                    if t <= pos and t < total:
                        stats[h, 4 if t < old else 5] += 1
                        if t < history:
                            frequencies[h, t] += 1
                            canonical[h, t] = min(canonical[h, t], origin * bs + o)
    # Compaction of nonempty private slots (query_private.py:108-128).
    counts = np.zeros(heads, np.int32)
    active_keys = np.full((heads, cap), INT32_MAX, np.int64)
    required = np.zeros((heads, cap), np.int64)
    private_mapping = np.full((heads, cap), -1, np.int64)
    keys = []
    for h in range(heads):
        rank = 0
        for i in range(cap):
            if private_required[h, i] > 0:
                active_keys[h, rank] = private_keys[h, i]
                required[h, rank] = private_required[h, i]
                private_mapping[h, i] = rank
                rank += 1
        counts[h] = rank
        keys.append([int(k) for k in active_keys[h, :rank]])
    region_counts = np.zeros(len(bases), np.int64)
    address, hbm, slots, valid, starts, flags = _resolve(
        geo, keys, counts, required, desc, tags, locs, host_locs, hot_data, bases,
        pool_tokens, page_size, stats, region_counts, hbm_locs)
    rows = q_count * heads
    all_ids = np.full((rows, width), -1, np.int32)
    all_counts = np.zeros(rows, np.int32)
    row_positions = np.zeros(rows, np.int64)
    for q in range(q_count):
        for h in range(heads):
            r = q * heads + h
            row_positions[r] = positions[q]
            if stats[h, 6]:
                continue
            n_valid = 0
            for i in range(width):
                origin = int(occurrences[q, h, i])
                if origin < 0:
                    continue
                compact = int(private_mapping[h, origin])
                if compact < 0:
                    continue
                all_ids[r, n_valid] = h * cap + compact
                n_valid += 1
            all_counts[r] = n_valid
    if consumer_ctas is None:
        consumer_ctas = min(rows, 256)
    if read_order == "physical":
        ioids, ranks, missing = physical_order(flags)
        first = near = None
    else:
        ioids, ranks, missing, first, near, _ = consumption_order(
            all_ids, all_counts, row_positions, flags, consumer_ctas, width,
            shared=read_order == "consumption_depth_shared")
    chosen = hot_choice(frequencies, hot)
    return dict(
        geometry=geo, active_counts=counts, active_keys=active_keys,
        required=required, stats=stats, address=address, hbm=hbm,
        slots=slots.reshape(-1), valid=valid, starts=starts, flags=flags,
        region_counts=region_counts, all_ids=all_ids, all_counts=all_counts,
        positions=row_positions, ioids=ioids, ranks=ranks, missing=missing,
        first_depth=first, near=near, frequencies=frequencies, chosen=chosen,
        canonical=canonical, private_mapping=private_mapping,
        consumer_ctas=consumer_ctas,
    )
