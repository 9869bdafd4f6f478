"""One NSA extend layer, in float64 or in the reference's bf16 sequence (test oracle).

Given one layer's input hidden states, its weights, the user's stored
history K/V for that layer (read back from the backing pool by the caller)
and the block selections the device made for the layer, this computes the
layer's output hidden states, either in exact arithmetic (float64) or with
the reference model's bf16 rounding sequence:

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
import torch.nn.functional as F

F64 = torch.float64


def _norm(x, weight, eps, acc):
    """RMSNorm as the reference computes it (models/tensor_ops.py): the
    statistics in the accumulation type, the result in x's type, then the
    gain."""
    value = x.to(acc)
    normalized = value * torch.rsqrt(value.square().mean(-1, keepdim=True) + eps)
    return normalized.to(x.dtype) * weight


def _rotate(x, positions, theta, acc):
    """Rotate-half RoPE; the phase in the accumulation type, cos / sin and the
    products in x's type (models/tensor_ops.py rotary)."""
    dim = x.shape[-1]
    inv = 1.0 / theta ** (torch.arange(0, dim, 2, device=x.device, dtype=acc) / dim)
    phase = positions.to(acc)[:, None] * inv[None, :]
    phase = torch.cat((phase, phase), -1)
    cos, sin = phase.cos().to(x.dtype)[:, None, :], phase.sin().to(x.dtype)[:, None, :]
    left, right = x[..., : dim // 2], x[..., dim // 2:]
    return x * cos + torch.cat((-right, left), -1) * sin


def _attend(q, k, v, mask, acc):
    """q [R, H, G, d], k / v [R, H, S, d] per row (or [S, H, d] shared),
    mask [R, S] or [R, H, S] -> [R, H, G, d] in q's type, computed in the
    accumulation type; a row with nothing visible gets 0."""
    scale = q.shape[-1] ** -0.5
    q, k, v = q.to(acc), k.to(acc), v.to(acc)
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
    length) of sequence [T, H, 128]: for K and V, W2 silu(W1 vec(x + pe)),
    every step in the sequence's type."""
    total, heads, width = sequence.shape
    d = width // 2
    count = (total - length) // stride + 1 if total >= length else 0
    if not count:
        return sequence.new_zeros(0, heads, width)
    windows = sequence.unfold(0, length, stride).permute(0, 1, 3, 2)  # [C, H, l, 128]
    parts = []
    for i, lo in enumerate((0, d)):
        x = windows[..., lo: lo + d] + w["cmp_pe"][i]
        hid = F.silu(F.linear(x.reshape(count, heads, length * d), w["cmp_w1"][i]))
        parts.append(F.linear(hid, w["cmp_w2"][i]))
    return torch.cat(parts, -1)


def _tokens_of(blocks, positions, bs):
    """Token ids [R, H, n * bs] of each row's selected blocks and their mask
    (a token counts if its block is >= 0 and it is at or before the row)."""
    offsets = torch.arange(bs, device=blocks.device)
    tokens = (blocks.clamp(min=0)[..., None] * bs + offsets).flatten(2)
    keep = (blocks >= 0)[..., None].expand(*blocks.shape, bs).flatten(2)
    keep = keep & (tokens <= positions[:, None, None])
    return tokens, keep


PRECISIONS = {"f64": (F64, F64), "bf16": (torch.bfloat16, torch.float32)}


def extend_layer(hidden, weights, history, positions, blocks, *, q_heads, kv_heads, head_dim,
                 block_size, window, rope_theta=10000.0, eps=1e-6, compression="mean",
                 cmp_block=32, cmp_stride=16, row_chunk=64, precision="f64",
                 return_records=False, trace=False):
    """One candidate's rows through one layer.

    hidden [R, D] (any float dtype; the layer input), history [old, H, 128]
    (K || V of tokens 0 .. old - 1), positions [R] = old .. old + R - 1 (the
    rows are the tokens that follow the history, in order), blocks [R, H, n]
    true block ids (-1: unused slot) -> output [R, D].

    ``precision``: "f64" computes everything in float64 (exact arithmetic
    for these sizes); "bf16" follows the reference model's rounding sequence
    (``models/nsa/model.py:440-492``, ``models/tensor_ops.py``, the torch
    branch of ``ops.py``): every tensor, GEMM output and elementwise result
    rounded to bf16, attention scores / softmax / weighted sums in fp32 with
    bf16 outputs, gate mix as bf16 multiply and two addcmuls. With
    ``return_records`` the rows' own K || V [R, H, 128] comes back too; with
    ``trace`` a dict with "out", "records", "mixed" (the gated attention
    output [R, H, G, d]) and "branches" (compressed, selected, window).
    """
    dt, acc = PRECISIONS[precision]
    device = hidden.device
    w = {name: t.to(dt) for name, t in weights.items()}
    rows, groups, d = len(hidden), q_heads // kv_heads, head_dim
    positions = positions.to(device=device, dtype=torch.int64)
    h = hidden.to(dt)
    x = _norm(h, w["in_norm"], eps, acc)
    q = F.linear(x, w["q"]).view(rows, q_heads, d)
    k = F.linear(x, w["k"]).view(rows, kv_heads, d)
    v = F.linear(x, w["v"]).view(rows, kv_heads, d)
    gates = torch.sigmoid(F.linear(x, w["g"])).view(rows, kv_heads, groups, 3)
    q, k = _rotate(q, positions, rope_theta, acc), _rotate(k, positions, rope_theta, acc)
    q = q.reshape(rows, kv_heads, groups, d)
    sequence = torch.cat((history.to(device, dt), torch.cat((k, v), -1)))  # [T, H, 128]
    total = len(sequence)

    # Compressed branch.
    if compression == "mean":
        complete = total // block_size
        keys = sequence[: complete * block_size].view(complete, block_size, kv_heads, 2 * d)
        keys = keys.to(acc).mean(1).to(dt)
        ends = (torch.arange(complete, device=device) + 1) * block_size
    else:
        keys = _compress_windows(sequence, w, cmp_block, cmp_stride)
        ends = torch.arange(len(keys), device=device) * cmp_stride + cmp_block
    if len(keys):
        cmp = _attend(q, keys[..., :d], keys[..., d:],
                      ends[None, :] <= positions[:, None] + 1, acc).to(dt)
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
        slc[r] = _attend(q[r], gathered[..., :d], gathered[..., d:], keep, acc).to(dt)
        # Window (pos - W, pos].
        span = pos[:, None] - window + 1 + torch.arange(window, device=device)[None, :]
        visible = span >= 0
        near = sequence[span.clamp(min=0)].permute(0, 2, 1, 3)         # [r, H, W, 128]
        win[r] = _attend(q[r], near[..., :d], near[..., d:], visible, acc).to(dt)

    mixed = slc * gates[..., 1, None]
    mixed = torch.addcmul(mixed, cmp, gates[..., 0, None])
    mixed = torch.addcmul(mixed, win, gates[..., 2, None])
    h = h + F.linear(mixed.reshape(rows, -1), w["o"])
    x = _norm(h, w["post_norm"], eps, acc)
    out = h + F.linear(F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"]), w["down"])
    records = sequence[len(history):]
    if trace:
        return dict(out=out, records=records, mixed=mixed, branches=(cmp, slc, win))
    if return_records:  # this chunk's K || V, as a later chunk's history
        return out, records
    return out


def layer_agreement(got, want):
    """Per-row agreement of a device layer output with the oracle's:
    (max-abs difference, minimum row cosine)."""
    got, want = got.to(F64), want.to(F64)
    diff = float((got - want).abs().max())
    cos = torch.nn.functional.cosine_similarity(got, want, dim=-1)
    return diff, float(cos.min())
