"""One NSA extend layer in float64 (test oracle).

Given one layer's input hidden states, its weights, the user's stored
history K/V for that layer (read back from the backing pool by the caller)
and the block selections the device made for the layer, this computes the
layer's output hidden states with every step restated in exact arithmetic:

* RMSNorm, q/k/v/gate projections, rotary embedding, o_proj, RMSNorm and the
  SwiGLU FFN (``models/nsa/model.py:440-492``, ``models/tensor_ops.py``);
* the compressed branch over the complete compressed keys visible to each
  row: mean-pooled block summaries (``models/nsa/ops.py:62-70, 73-106``) or
  the NSA paper's MLP-compressed windows (the arithmetic of
  ``oracle/attention.py`` ``compress_mlp``, batched over windows; a
  restatement, not pinned to reference output);
* the selected branch: each row attends the tokens of its own selected
  blocks up to its position, duplicates kept
  (``models/nsa/backends/io_plan.py:291-331``);
* the sliding window over positions (pos - W, pos] (``ops.py:154-205``);
* the sigmoid gate mix of the three branches (``model.py:456-473``).

Only which blocks are selected is taken from the device: the top-n rule on
nearly equal scores could otherwise pick different blocks on the two sides.
The rule itself is checked separately, bit for bit on the device's own
scores. Nothing here sees a plan, a staging buffer, the hot replica or a
ready flag, so a per-layer match checks all of them.

Test infrastructure only: the product package never imports it.
"""

import torch

F64 = torch.float64


def _norm(x, weight, eps):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + eps) * weight.to(F64)


def _rotate(x, positions, theta):
    dim = x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, device=x.device, dtype=F64) / dim)
    phase = positions.to(F64)[:, None] * inv[None, :]
    phase = torch.cat((phase, phase), -1)[:, None, :]
    left, right = x[..., : dim // 2], x[..., dim // 2:]
    return x * phase.cos() + torch.cat((-right, left), -1) * phase.sin()


def _attend(q, k, v, mask):
    """q [R, H, G, d], k / v [R, H, S, d] per row (or [S, H, d] shared),
    mask [R, S] or [R, H, S] -> [R, H, G, d]; a row with nothing visible gets 0."""
    scale = q.shape[-1] ** -0.5
    if k.dim() == 3:
        logits = torch.einsum("rhgd,shd->rhgs", q, k) * scale
    else:
        logits = torch.einsum("rhgd,rhsd->rhgs", q, k) * scale
    if mask.dim() == 2:
        mask = mask[:, None, :]
    logits = logits.masked_fill(~mask[:, :, None, :], -torch.inf)
    prob = logits.softmax(-1).nan_to_num()
    if v.dim() == 3:
        return torch.einsum("rhgs,shd->rhgd", prob, v)
    return torch.einsum("rhgs,rhsd->rhgd", prob, v)


def _compress_windows(sequence, w, length, stride):
    """Keys [C, H, 128] of the complete windows [i * stride, i * stride +
    length) of sequence [T, H, 128]: for K and V, W2 silu(W1 vec(x + pe))."""
    total, heads, width = sequence.shape
    d = width // 2
    count = (total - length) // stride + 1 if total >= length else 0
    if not count:
        return sequence.new_zeros(0, heads, width)
    windows = sequence.unfold(0, length, stride).permute(0, 1, 3, 2)  # [C, H, l, 128]
    parts = []
    for i, lo in enumerate((0, d)):
        x = windows[..., lo: lo + d] + w["cmp_pe"][i]
        hid = torch.nn.functional.silu(x.reshape(count, heads, length * d) @ w["cmp_w1"][i].T)
        parts.append(hid @ w["cmp_w2"][i].T)
    return torch.cat(parts, -1)


def _tokens_of(blocks, positions, bs):
    """Token ids [R, H, n * bs] of each row's selected blocks and their mask
    (a token counts if its block is >= 0 and it is at or before the row)."""
    offsets = torch.arange(bs, device=blocks.device)
    tokens = (blocks.clamp(min=0)[..., None] * bs + offsets).flatten(2)
    keep = (blocks >= 0)[..., None].expand(*blocks.shape, bs).flatten(2)
    keep = keep & (tokens <= positions[:, None, None])
    return tokens, keep


def extend_layer(hidden, weights, history, positions, blocks, *, q_heads, kv_heads, head_dim,
                 block_size, window, rope_theta=10000.0, eps=1e-6, compression="mean",
                 cmp_block=32, cmp_stride=16, row_chunk=64, return_records=False):
    """One candidate's rows through one layer.

    hidden [R, D] (any float dtype; the layer input), history [old, H, 128]
    (K || V of tokens 0 .. old - 1), positions [R] = old .. old + R - 1 (the
    rows are the tokens that follow the history, in order), blocks [R, H, n]
    true block ids (-1: unused slot) -> output [R, D] float64 (and, with
    ``return_records``, the rows' own K || V [R, H, 128]).
    """
    device = hidden.device
    w = {name: t.to(F64) for name, t in weights.items()}
    rows, groups, d = len(hidden), q_heads // kv_heads, head_dim
    positions = positions.to(device=device, dtype=torch.int64)
    h = hidden.to(F64)
    x = _norm(h, w["in_norm"], eps)
    q = (x @ w["q"].T).view(rows, q_heads, d)
    k = (x @ w["k"].T).view(rows, kv_heads, d)
    v = (x @ w["v"].T).view(rows, kv_heads, d)
    gates = torch.sigmoid(x @ w["g"].T).view(rows, kv_heads, groups, 3)
    q, k = _rotate(q, positions, rope_theta), _rotate(k, positions, rope_theta)
    q = q.view(rows, kv_heads, groups, d)
    sequence = torch.cat((history.to(device, F64), torch.cat((k, v), -1)))  # [T, H, 128]
    total = len(sequence)

    # Compressed branch.
    if compression == "mean":
        complete = total // block_size
        keys = sequence[: complete * block_size].view(complete, block_size, kv_heads, 2 * d)
        keys = keys.mean(1)
        ends = (torch.arange(complete, device=device) + 1) * block_size
    else:
        keys = _compress_windows(sequence, w, cmp_block, cmp_stride)
        ends = torch.arange(len(keys), device=device) * cmp_stride + cmp_block
    if len(keys):
        cmp = _attend(q, keys[..., :d], keys[..., d:], ends[None, :] <= positions[:, None] + 1)
    else:
        cmp = torch.zeros_like(q)

    slc = torch.empty_like(q)
    win = torch.empty_like(q)
    blocks = blocks.to(device=device, dtype=torch.int64)
    for lo in range(0, rows, row_chunk):
        r = slice(lo, min(rows, lo + row_chunk))
        pos = positions[r]
        # Selected blocks: gather each row's tokens per KV head.
        tokens, keep = _tokens_of(blocks[r], pos, block_size)
        gathered = sequence[tokens.clamp(max=total - 1),  # masked tokens: any index
                            torch.arange(kv_heads, device=device)[None, :, None]]
        slc[r] = _attend(q[r], gathered[..., :d], gathered[..., d:], keep)
        # Window (pos - W, pos].
        span = pos[:, None] - window + 1 + torch.arange(window, device=device)[None, :]
        visible = span >= 0
        near = sequence[span.clamp(min=0)]                              # [r, W, H, 128]
        near = near.permute(0, 2, 1, 3)
        win[r] = _attend(q[r], near[..., :d], near[..., d:], visible)

    mixed = slc * gates[..., 1, None] + cmp * gates[..., 0, None] + win * gates[..., 2, None]
    h = h + mixed.reshape(rows, -1) @ w["o"].T
    x = _norm(h, w["post_norm"], eps)
    ffn = torch.nn.functional.silu(x @ w["gate"].T) * (x @ w["up"].T)
    out = h + ffn @ w["down"].T
    if return_records:  # this chunk's K || V, as a later chunk's history
        return out, sequence[len(history):]
    return out


def layer_agreement(got, want):
    """Per-row agreement of a device layer output with the oracle's:
    (max-abs difference, minimum row cosine)."""
    got, want = got.to(F64), want.to(F64)
    diff = float((got - want).abs().max())
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    return diff, float(cos.min())
