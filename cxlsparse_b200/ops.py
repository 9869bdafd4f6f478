"""NSA local branches on the device: compressed attention + top-n selection.

Mirrors ``cxl_recsys/models/nsa/ops.py`` / ``fla.py``:
``compressed_attention_select(query, compressed, positions, total, block_size,
count)`` returns ``(output [Q, H, G, 64] bf16, blocks [Q, H, width] int32)``
with width = min(count, ceil(total / block_size)) (fla.py:6-62), and
``append_compressed`` mean-pools complete blocks (ops.py:62-70). The window
branch and the gate mix run inside the transport's fetch/attend launch.
"""

import torch

from . import _lib


def select_geometry(queries, heads, summaries, total, block_size, count, *, segments=None,
                    window=None, stride=None, forced=False):
    """The C geometry of one compressed-select call (see ``cxs_select_geometry``)."""
    segment_start, segment_tokens = segments or (0, 0)
    return _lib.SelectGeometry(
        queries=queries, heads=heads, block_size=block_size, count=count, summaries=summaries,
        window=window or block_size, stride=stride or block_size, forced=int(bool(forced)),
        total=total, segment_start=segment_start, segment_tokens=segment_tokens)


def score_columns(geometry):
    """Columns of the block-score output for ``geometry``."""
    columns = _lib.c_i32(0)
    _lib.check(_lib.lib().cxs_select_score_columns(geometry, columns))
    return columns.value


def compressed_attention_select(query, compressed, positions, total, block_size, count, *,
                                scores=None, segments=None, window=None, stride=None,
                                forced=False):
    """Compressed-token attention and top-n block ids; ``scores`` optionally
    receives the [Q, H, columns] fp32 block scores the selection was made
    from (columns = C in the reference geometry, see ``score_columns``).
    ``segments=(segment_start, segment_tokens)`` selects over candidate
    segments (positions, summaries and returned block ids in the segment
    layout of ``cxs_attend_geometry``; ``total`` is one candidate's true
    history + suffix length). ``window`` / ``stride`` (default: the block
    size, the reference's mean-pooled summaries) describe overlapping
    compressed keys; ``forced`` adds the previous block and block 0 after
    the current one (the NSA paper's geometry, Yuan et al. 2025)."""
    queries, heads, groups, dim = query.shape
    if groups != 16 or dim != 64 or query.dtype != torch.bfloat16:
        raise ValueError("query must be bf16 [Q, H, 16, 64]")
    if compressed.ndim != 3 or compressed.shape[1:] != (heads, 128):
        raise ValueError("compressed must be [C, H, 128] (K || V)")
    query = query.contiguous()
    compressed = compressed.contiguous()
    positions = positions.to(torch.int32).contiguous()
    width = min(count, (total + block_size - 1) // block_size)
    output = torch.empty_like(query)
    blocks = torch.empty((queries, heads, width), dtype=torch.int32, device=query.device)
    geometry = select_geometry(queries, heads, len(compressed), total, block_size, count,
                               segments=segments, window=window, stride=stride, forced=forced)
    if scores is not None and scores.shape != (queries, heads, score_columns(geometry)):
        raise ValueError("scores must be [Q, H, score_columns] fp32")
    stream = torch.cuda.current_stream(query.device)
    _lib.check(_lib.lib().cxs_compressed_select_nsa(
        geometry, query.data_ptr(), compressed.data_ptr() if len(compressed) else None,
        positions.data_ptr(), output.data_ptr(), blocks.data_ptr(), _lib.ptr(scores),
        stream.cuda_stream))
    return output, blocks


def block_summaries(tokens, block_size):
    """Mean of each complete block of ``tokens`` [n, H, 128] -> [n // BS, H, 128]."""
    tokens = tokens.contiguous()
    count = len(tokens) // block_size
    out = torch.empty((count, *tokens.shape[1:]), dtype=tokens.dtype, device=tokens.device)
    if count:
        stream = torch.cuda.current_stream(tokens.device)
        _lib.check(_lib.lib().cxs_block_summaries(tokens.data_ptr(), len(tokens),
                                                  tokens.shape[1], block_size, out.data_ptr(),
                                                  stream.cuda_stream))
    return out


def block_summaries_segments(tokens, count, block_size, out, segments, token_stride,
                             summary_stride):
    """Summaries of ``segments`` runs of ``count`` records in one launch: run s
    pools tokens[s * token_stride :][:count] into out[s * summary_stride :]
    (tokens / out are [n, H, 128] bf16 buffers, written in place)."""
    if count // block_size:
        stream = torch.cuda.current_stream(tokens.device)
        _lib.check(_lib.lib().cxs_block_summaries_segments(
            tokens.data_ptr(), count, tokens.shape[1], block_size, out.data_ptr(), segments,
            token_stride, summary_stride, stream.cuda_stream))


def append_compressed(compressed, tail, current, block_size):
    """(summaries + new complete blocks of tail||current, new tail) (ops.py:62-70)."""
    values = torch.cat((tail, current))
    count = len(values) // block_size
    added = block_summaries(values[: count * block_size], block_size)
    return torch.cat((compressed, added)), values[count * block_size:].clone()
