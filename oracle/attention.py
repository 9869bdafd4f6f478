"""CPU restatement of the NSA branch arithmetic (test oracle and CPU baseline).

* ``selected_attention``: FP64 dense softmax over each row's selected tokens,
  duplicates kept (``models/nsa/backends/io_plan.py:291-331``).
* ``compressed_attention_select``: compressed-token attention plus top-n block
  selection (``models/nsa/ops.py:73-123``), fp32.
* ``window_attention``: sliding window over the retained window + suffix KV
  (``models/nsa/ops.py:154-205``, CPU branch), fp32.
* ``append_compressed``: mean-pooled block summaries (``models/nsa/ops.py:62-70``).
* ``gate_mix``: the sigmoid-gate combination in the reference's BF16 rounding
  sequence (``models/nsa/model.py:470-473``).
* ``topn_from_scores``: the ordering rule alone, for bit-exact checks of a
  device selection against its own exported scores.
* ``compress_mlp``, ``block_scores``, ``topn_forced``, ``compressed_select_nsa``:
  the NSA paper's selection geometry (overlapping MLP-compressed windows,
  aggregated block scores, forced blocks), which the reference does not have:
  a restatement of the published NSA method, not pinned to reference output.

Test infrastructure only: the product path never imports this package.
"""

import torch


def selected_attention(query, backing, blocks, positions, bs):
    """query [Q,H,G,64], backing [T,H,128], blocks [Q,H,W] -> FP64 [Q,H,G,64]."""
    queries, heads, width = blocks.shape
    out = torch.zeros(query.shape, dtype=torch.float64)
    for q in range(queries):
        pos = int(positions[q])
        for h in range(heads):
            tokens = []
            for b in blocks[q, h].tolist():
                if b < 0 or pos < 0:
                    continue
                start = b * bs
                stop = min(start + bs, pos + 1)
                tokens.extend(range(start, stop))
            if tokens:
                kv = backing[tokens, h].double()
                scores = (query[q, h].double() @ kv[:, :64].T) * (64 ** -0.5)
                out[q, h] = scores.softmax(-1) @ kv[:, 64:]
    return out


def topn_from_scores(scores, positions, bs, count, total):
    """Ordering rule of the top-n selection (ops.py:107-123).

    ``scores`` [Q,H,C] fp32 summed GQA probabilities over complete compressed
    blocks. Blocks after the current one are invisible, the current block
    always ranks first, ties go to the lower block id (stable), and entries
    after the current block become -1.
    """
    queries, heads = scores.shape[:2]
    blocks = (total + bs - 1) // bs
    width = min(count, blocks)
    padded = torch.full((queries, heads, blocks), 0.0, dtype=torch.float32)
    n = min(blocks, scores.shape[2])
    padded[..., :n] = scores[..., :n].float()
    current = torch.as_tensor(positions) // bs
    causal = torch.arange(blocks)[None, None, :] <= current[:, None, None]
    padded.masked_fill_(~causal, -torch.inf)
    padded.scatter_(2, current[:, None, None].expand(-1, heads, 1), torch.inf)
    selected = padded.argsort(dim=-1, descending=True, stable=True)[..., :width]
    selected.masked_fill_(selected > current[:, None, None], -1)
    return selected


def compressed_attention_select(query, key, value, positions, total, bs, count):
    """Q [Q,H,G,D], compressed K/V [C,H,D] -> (output [Q,H,G,D] fp32, blocks, scores)."""
    queries, heads, groups, dim = query.shape
    positions = torch.as_tensor(positions)
    c = len(key)
    if c:
        logits = torch.einsum("qhgd,chd->qhgc", query.float(), key.float()) * dim ** -0.5
        mask = (torch.arange(c) + 1) * bs <= positions[:, None] + 1
        logits.masked_fill_(~mask[:, None, None, :], -torch.inf)
        probability = logits.softmax(-1).nan_to_num()
        output = torch.einsum("qhgc,chd->qhgd", probability, value.float())
        scores = probability.sum(2)
    else:
        output = torch.zeros(query.shape, dtype=torch.float32)
        scores = torch.zeros((queries, heads, 0))
    selected = topn_from_scores(scores, positions, bs, count, total)
    return output, selected, scores


def window_attention(query, records, positions, start, window):
    """Tokens (pos-W, pos] of ``records`` (logical index = local + start), fp32."""
    queries, heads, groups, dim = query.shape
    out = torch.zeros(query.shape, dtype=torch.float32)
    for q in range(queries):
        pos = int(positions[q])
        if pos < 0:
            continue
        lo = max(0, pos - window + 1)
        local = torch.arange(lo, pos + 1) - start
        local = local[(local >= 0) & (local < len(records))]
        if not len(local):
            continue
        kv = records[local].float()
        for h in range(heads):
            scores = (query[q, h].float() @ kv[:, h, :dim].T) * dim ** -0.5
            out[q, h] = scores.softmax(-1) @ kv[:, h, dim:]
    return out


def append_compressed(compressed, tail, current, bs):
    """Mean-pool complete BS-token blocks of tail+current (ops.py:62-70)."""
    values = torch.cat((tail, current))
    count = len(values) // bs
    added = values[: count * bs].reshape(count, bs, *values.shape[1:]).float().mean(1)
    return torch.cat((compressed, added.to(values.dtype))), values[count * bs:].clone()


def gate_mix(selected, compressed, window, gates):
    """bf16 mul / addcmul / addcmul sequence; gates [..., 3] = (cmp, slc, win)."""
    mixed = selected * gates[..., 1, None]
    mixed = torch.addcmul(mixed, compressed, gates[..., 0, None])
    return torch.addcmul(mixed, window, gates[..., 2, None])


# ---------------------------------------------------------------------------
# The NSA paper's selection geometry (Yuan et al. 2025; not in the reference, which uses
# mean-pooled summaries with block = stride = selection block and only the
# current block forced): overlapping compression windows of `l` tokens at
# stride `d` mapped to one key/value each by an MLP, selection-block scores
# aggregated from the overlapping compressed scores, and top-n with block 0
# and the two local blocks forced. Restated from the published NSA method
# (Yuan et al. 2025, "Native Sparse Attention": token compression with a
# learnable MLP and intra-block position encoding; selection scores derived
# from the compression-attention scores, weighted by how many stride steps of
# a compressed window fall into a selection block; GQA heads of a group
# share the selection by summing their scores).
# ---------------------------------------------------------------------------


def compress_mlp(records, weights, l, d, *, bf16_steps=False):
    """records [T, H, 128] (K || V) -> [C, H, 128] for the complete windows
    [i*d, i*d + l), C = (T - l) // d + 1. ``weights`` holds, for K and V,
    pe [l, 64], w1 [hidden, l*64], w2 [64, hidden]: phi(x) = w2 silu(w1
    vec(x + pe)), computed in fp32 and rounded to bf16 once, or, with
    ``bf16_steps``, rounded to bf16 after the position add, w1 and the silu as
    a bf16 model computes it."""
    t, heads = records.shape[:2]
    count = (t - l) // d + 1 if t >= l else 0
    out = torch.zeros(count, heads, 128, device=records.device)

    def step(x):
        return x.bfloat16().float() if bf16_steps else x

    for part, lo in (("k", 0), ("v", 64)):
        pe, w1, w2 = (weights[f"{part}_{n}"].float() for n in ("pe", "w1", "w2"))
        for i in range(count):
            x = step(records[i * d: i * d + l, :, lo: lo + 64].float() + pe[:, None, :])
            x = x.permute(1, 0, 2).reshape(heads, l * 64)
            hidden = step(torch.nn.functional.silu(step(x @ w1.T)))
            out[i, :, lo: lo + 64] = hidden @ w2.T
    return out.to(records.dtype)


def overlap_weight(i, j, l, d, bs):
    """Stride steps of compressed window i ([i*d, i*d + l)) inside selection
    block j ([j*bs, (j+1)*bs)): the NSA aggregation weight."""
    lo, hi = max(i * d, j * bs), min(i * d + l, (j + 1) * bs)
    return max(0, hi - lo) // d


def block_scores(key_scores, l, d, bs, blocks):
    """[..., C] summed compressed probabilities -> [..., blocks] selection
    scores, each the weighted sum over the windows overlapping the block in
    ascending window order. With l = d = bs this is the identity."""
    c = key_scores.shape[-1]
    out = torch.zeros(*key_scores.shape[:-1], blocks, dtype=key_scores.dtype)
    for j in range(blocks):
        first = max(0, -(-(j * bs - l + 1) // d))
        last = min(c - 1, ((j + 1) * bs - 1) // d)
        for i in range(first, last + 1):
            w = overlap_weight(i, j, l, d, bs)
            if w:
                out[..., j] += w * key_scores[..., i]
    return out


def topn_forced(scores, positions, bs, count, total, forced):
    """Selection order over block scores [Q, H, B]: the current block, then
    (``forced``) the previous block and block 0, then the other blocks before
    the current one by score descending, ties to the lower id; width =
    min(count, ceil(total / bs)); missing entries -1. Without ``forced`` this
    is the reference rule (``topn_from_scores``)."""
    queries, heads, _ = scores.shape
    width = min(count, -(-total // bs))
    out = torch.full((queries, heads, width), -1, dtype=torch.int64)
    for q in range(queries):
        current = int(positions[q]) // bs
        for h in range(heads):
            picks = [current]
            if forced:
                for b in (current - 1, 0):
                    if 0 <= b < current and b not in picks:
                        picks.append(b)
            rest = [b for b in range(current) if b not in picks]
            rest.sort(key=lambda b: (-float(scores[q, h, b]), b))
            picks = (picks + rest)[:width]
            out[q, h, : len(picks)] = torch.tensor(picks)
    return out


def compressed_select_nsa(query, keys, positions, total, bs, count, l, d, forced):
    """Compressed attention over the complete windows visible to each row
    (i*d + l <= pos + 1) and top-n over the aggregated block scores.
    query [Q, H, G, 64], keys [C, H, 128] -> (output fp32, blocks, block scores)."""
    queries, heads, groups, dim = query.shape
    positions = torch.as_tensor(positions)
    c = len(keys)
    blocks_n = -(-total // bs)
    if c:
        logits = torch.einsum("qhgd,chd->qhgc", query.float(), keys[:, :, :64].float()) * dim ** -0.5
        ends = torch.arange(c) * d + l
        mask = ends[None, :] <= positions[:, None] + 1
        logits.masked_fill_(~mask[:, None, None, :], -torch.inf)
        probability = logits.softmax(-1).nan_to_num()
        output = torch.einsum("qhgc,chd->qhgd", probability, keys[:, :, 64:].float())
        key_scores = probability.sum(2)
    else:
        output = torch.zeros(query.shape)
        key_scores = torch.zeros(queries, heads, 0)
    scores = block_scores(key_scores, l, d, bs, blocks_n)
    return output, topn_forced(scores, positions, bs, count, total, forced), scores
