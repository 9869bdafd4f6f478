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
