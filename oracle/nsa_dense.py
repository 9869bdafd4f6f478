"""Dense resident NSA forward (test oracle).

When a sequence's causal blocks all fit in the selection (history + suffix <=
top-n x block size), the selected branch of NSA attends to every earlier
token, so the whole model reduces to three dense branches per layer:
compressed-token attention, full causal attention and the sliding window,
mixed by the sigmoid gates. This module computes that directly with torch, on
any device, following the structure of the reference's independent dense
oracle (tests/test_nsa.py:152-236: bf16 activations, fp32 attention
arithmetic, GQA by repeating the KV heads) with this model's geometry
(selection block, window, compression). It never sees a block table, a plan,
a pool or a cache, so it checks all of them at once.

Pinned: with mean-pooled compression it is bit-identical to the reference's
own dense oracle (run on CPU into tests/golden/dense_model.npz; checked by
tests/test_oracle_golden.py). The MLP-compression branch restates the NSA
paper's compression (oracle/attention.py compress_mlp) and is not pinned.

Test infrastructure only: the product package never imports it.
"""

import torch
import torch.nn.functional as F

from .attention import compress_mlp


def _norm(x, weight, eps):
    return (x.float() * (x.float().square().mean(-1, keepdim=True) + eps).rsqrt()
            ).to(x.dtype) * weight


def _attention(q, k, v, mask, groups):
    """q [T, Hq, D], k / v [S, Hkv, D], mask [T, S] -> [T, Hq, D] bf16."""
    dim = q.shape[-1]
    score = torch.einsum("qhd,khd->hqk", q.float(),
                         k.repeat_interleave(groups, 1).float()) / dim ** 0.5
    probability = score.masked_fill(~mask, -torch.inf).softmax(-1).nan_to_num()
    return torch.einsum("hqk,khd->qhd", probability,
                        v.repeat_interleave(groups, 1).float()).to(q.dtype)


def dense_forward(token_ids, embed, layers, final_norm, *, q_heads, kv_heads, head_dim,
                  block_size, window, rope_theta=10000.0, eps=1e-6, compression="mean",
                  cmp_block=32, cmp_stride=16):
    """Final hidden states [T, hidden] of the whole sequence `token_ids` from
    position 0. `layers[i]` holds the projection weights q, k, v, g, o, gate,
    up, down, in_norm, post_norm (and cmp_pe, cmp_w1, cmp_w2 stacked [K, V]
    for compression="mlp")."""
    device = embed.device
    hidden = F.embedding(token_ids.to(device), embed)
    length, dim, groups = len(token_ids), head_dim, q_heads // kv_heads
    pos = torch.arange(length, device=device)
    # position / theta^(i/d), divided rather than multiplied by an inverse
    # frequency: that is the reference oracle's rounding (the bf16 sine table
    # differs in a few entries otherwise), which keeps the two bit-identical.
    freq = rope_theta ** (torch.arange(0, dim, 2, device=device).float() / dim)
    phase = pos.float()[:, None] / freq[None, :]
    phase = torch.cat((phase, phase), -1)[:, None]
    cos, sin = phase.cos().to(hidden.dtype), phase.sin().to(hidden.dtype)
    causal = pos[None] <= pos[:, None]
    for w in layers:
        x = _norm(hidden, w["in_norm"], eps)
        q = F.linear(x, w["q"]).view(length, q_heads, dim)
        k = F.linear(x, w["k"]).view(length, kv_heads, dim)
        v = F.linear(x, w["v"]).view(length, kv_heads, dim)
        q, k = [a * cos + torch.cat((-a[..., dim // 2:], a[..., :dim // 2]), -1) * sin
                for a in (q, k)]
        gates = F.linear(x, w["g"]).view(length, q_heads, 3).sigmoid()
        if compression == "mean":
            complete = length // block_size
            ck = k[:complete * block_size].reshape(complete, block_size, kv_heads, dim)
            cv = v[:complete * block_size].reshape(complete, block_size, kv_heads, dim)
            ck, cv = ck.float().mean(1).to(k.dtype), cv.float().mean(1).to(v.dtype)
            ends = (torch.arange(complete, device=device) + 1) * block_size
        else:
            records = torch.cat((k, v), -1)
            weights = {f"{part}_{name}": w[f"cmp_{name}"][i]
                       for i, part in enumerate("kv") for name in ("pe", "w1", "w2")}
            keys = compress_mlp(records, weights, cmp_block, cmp_stride, bf16_steps=True)
            complete = len(keys)
            ck, cv = keys[..., :dim], keys[..., dim:]
            ends = torch.arange(complete, device=device) * cmp_stride + cmp_block
        cmp = (_attention(q, ck, cv, ends[None, :] <= pos[:, None] + 1, groups) if complete
               else torch.zeros_like(q))
        slc = _attention(q, k, v, causal, groups)
        win = _attention(q, k, v, causal & (pos[None] > pos[:, None] - window), groups)
        mixed = torch.addcmul(slc * gates[..., 1, None], cmp, gates[..., 0, None])
        mixed = torch.addcmul(mixed, win, gates[..., 2, None])
        hidden = hidden + F.linear(mixed.flatten(1), w["o"])
        x = _norm(hidden, w["post_norm"], eps)
        hidden = hidden + F.linear(F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"]),
                                   w["down"])
    return _norm(hidden, final_norm, eps)
