"""CPU restatement of the reference's torch NSA extend path (timed baseline only).

The reference's CPU route for one NSA layer is ``ops.local_branches(...,
backend="torch")`` (compressed attention + top-n selection + window,
``models/nsa/ops.py:12-59, 73-123, 154-205``), ``ops.indexed_attention`` for
the selected branch (``ops.py:132-151``) and the gate mix / o_proj / FFN of
``models/nsa/model.py:440-492``. This module runs that arithmetic in fp32 with
torch on the host cores, vectorised the same way (per-tile bmm). It is test
infrastructure: ``bench.py`` times it as the CPU baseline and as the
``--impl reference`` arm; the product package never imports it.

Pinned: on one seeded layer, ``CPUExtendPath.layer`` reproduces the output of
the reference's own CPU route (its ``_project``, ``local_branches(...,
backend="torch")``, ``indexed_attention`` and ``_finish``, run into
tests/golden/cpu_layer.npz) within 1e-5, and its selected tokens exactly
(tests/test_cpu_port_pinned.py).

For timing, history K/V, summaries and windows are seeded N(0, 1) stand-ins
of the right shapes: throughput does not depend on their values.
"""

import time

import torch


def rms_norm(x, weight, eps=1e-6):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * weight


def rotary(q, k, positions, inv_freq):
    freq = positions.float()[:, None] * inv_freq[None, :]
    phase = torch.cat((freq, freq), -1)
    cos, sin = phase.cos()[:, None, :], phase.sin()[:, None, :]

    def rotate(v):
        left, right = v.chunk(2, -1)
        return v * cos + torch.cat((-right, left), -1) * sin

    return rotate(q), rotate(k)


def indexed_attention(query, records, indices, tile=128):
    """query [R, G, D], records [T, 2D], indices [R, N] (-1 masked) (ops.py:132-151)."""
    out = torch.empty_like(query)
    dim = query.shape[-1]
    for begin in range(0, len(query), tile):
        end = min(begin + tile, len(query))
        ids = indices[begin:end]
        key, value = records[ids.clamp_min(0)].split(dim, -1)
        scores = torch.bmm(query[begin:end], key.transpose(1, 2)) * dim ** -0.5
        scores.masked_fill_(ids[:, None, :] < 0, -torch.inf)
        out[begin:end] = torch.bmm(scores.softmax(-1).nan_to_num(), value)
    return out


def compressed_select(query, keys, values, positions, total, bs, count):
    """ops.py:73-123 (torch branch)."""
    queries, heads, groups, dim = query.shape
    blocks = (total + bs - 1) // bs
    width = min(count, blocks)
    logits = torch.einsum("qhgd,chd->qhgc", query, keys) * dim ** -0.5
    valid = (torch.arange(len(keys)) + 1) * bs
    mask = valid[None, :] <= positions[:, None] + 1
    logits.masked_fill_(~mask[:, None, None, :], -torch.inf)
    probability = logits.softmax(-1).nan_to_num()
    output = torch.einsum("qhgc,chd->qhgd", probability, values)
    scores = torch.nn.functional.pad(probability.sum(2), (0, blocks - len(keys)))
    current = positions // bs
    causal = torch.arange(blocks)[None, None, :] <= current[:, None, None]
    scores.masked_fill_(~causal, -torch.inf)
    scores.scatter_(2, current[:, None, None].expand(-1, heads, 1), torch.inf)
    selected = scores.argsort(dim=-1, descending=True, stable=True)[..., :width]
    selected.masked_fill_(selected > current[:, None, None], -1)
    return output, selected


class CPUExtendPath:
    """fp32 NSA extend forward on the host: the reference CPU baseline."""

    def __init__(self, *, layers=16, hidden=2048, q_heads=32, kv_heads=2, head_dim=64,
                 ffn=5632, history=16384, block_size=64, block_counts=16, window=512,
                 seed=0):
        g = torch.Generator().manual_seed(seed)
        self.layers, self.hidden, self.kv_heads = layers, hidden, kv_heads
        self.q_heads, self.head_dim, self.groups = q_heads, head_dim, q_heads // kv_heads
        self.history, self.bs, self.count, self.window = history, block_size, block_counts, window

        def normal(*shape):
            return torch.randn(*shape, generator=g) * 0.02

        kvd = kv_heads * head_dim
        self.weights = [dict(q=normal(q_heads * head_dim, hidden), k=normal(kvd, hidden),
                             v=normal(kvd, hidden), g=normal(q_heads * 3, hidden),
                             o=normal(hidden, q_heads * head_dim), gate=normal(ffn, hidden),
                             up=normal(ffn, hidden), down=normal(hidden, ffn))
                        for _ in range(layers)]
        self.norm = torch.ones(hidden)
        # Per-layer history K/V in the backing pool, its summaries and window.
        self.kv = [torch.randn(history, kv_heads, 2 * head_dim, generator=g)
                   for _ in range(layers)]
        self.summaries = [kv.reshape(-1, block_size, kv_heads, 2 * head_dim).mean(1)
                          for kv in self.kv]
        self.inv_freq = 1.0 / (10000.0 ** (torch.arange(0, head_dim, 2).float() / head_dim))

    def layer(self, index, hidden, positions):
        w, H, E = self.weights[index], self.history, len(hidden)
        x = rms_norm(hidden, self.norm)
        q = (x @ w["q"].T).view(E, self.q_heads, self.head_dim)
        k = (x @ w["k"].T).view(E, self.kv_heads, self.head_dim)
        v = (x @ w["v"].T).view(E, self.kv_heads, self.head_dim)
        gates = torch.sigmoid(x @ w["g"].T).view(E, self.kv_heads, self.groups, 3)
        q, k = rotary(q, k, positions, self.inv_freq)
        query = q.view(E, self.kv_heads, self.groups, self.head_dim)
        current = torch.cat((k, v), -1)
        records = torch.cat((self.kv[index], current))          # history + suffix
        complete = (H + E) // self.bs
        summaries = torch.cat((self.summaries[index],
                               current[: (complete * self.bs - H)].reshape(
                                   -1, self.bs, self.kv_heads, 2 * self.head_dim).mean(1)))
        key, value = summaries.split(self.head_dim, -1)
        compressed, selected = compressed_select(query, key, value, positions, H + E, self.bs,
                                                 self.count)
        # Selected branch: expand blocks to token ids (ops.py:126-129), indexed attention.
        offsets = torch.arange(self.bs)
        tokens = (selected[..., None] * self.bs + offsets).flatten(-2)
        tokens = tokens.masked_fill((tokens < 0) | (tokens > positions[:, None, None]), -1)
        flat_records = records.reshape(-1, 2 * self.head_dim)           # [(T*H), 128]
        head_ids = torch.arange(self.kv_heads)[None, :, None]
        indices = torch.where(tokens >= 0, tokens * self.kv_heads + head_ids, -1)
        sel = indexed_attention(query.reshape(E * self.kv_heads, self.groups, self.head_dim),
                                flat_records, indices.reshape(E * self.kv_heads, -1))
        sel = sel.view_as(query)
        # Window branch (ops.py:194-205).
        window_offsets = torch.arange(1 - self.window, 1)
        logical = positions[:, None] + window_offsets
        win_idx = logical[:, None, :] * self.kv_heads + head_ids
        win_idx = win_idx.masked_fill((logical < 0)[:, None, :], -1)
        win = indexed_attention(query.reshape(E * self.kv_heads, self.groups, self.head_dim),
                                flat_records, win_idx.reshape(E * self.kv_heads, -1))
        win = win.view_as(query)
        mixed = sel * gates[..., 1, None] + compressed * gates[..., 0, None] + \
            win * gates[..., 2, None]
        hidden = hidden + mixed.reshape(E, -1) @ w["o"].T
        x = rms_norm(hidden, self.norm)
        mlp = torch.nn.functional.silu(x @ w["gate"].T) * (x @ w["up"].T)
        return hidden + mlp @ w["down"].T

    def forward(self, hidden, layers=None):
        positions = torch.arange(self.history, self.history + len(hidden))
        for index in range(layers or self.layers):
            hidden = self.layer(index, hidden, positions)
        return hidden


def time_cpu_extend(*, extend=256, history=16384, layers=16, steps=1, warmup=0,
                    threads=None, seed=0):
    """Median seconds per full extend forward on the host; returns (seconds, cores)."""
    threads = threads or torch.get_num_threads()
    torch.set_num_threads(threads)
    path = CPUExtendPath(layers=layers, history=history, seed=seed)
    hidden = torch.randn(extend, path.hidden, generator=torch.Generator().manual_seed(seed + 1))
    with torch.inference_mode():
        for _ in range(warmup):
            path.forward(hidden)
        times = []
        for _ in range(max(1, steps)):
            t0 = time.perf_counter()
            path.forward(hidden)
            times.append(time.perf_counter() - t0)
    times.sort()
    return times[len(times) // 2], threads
