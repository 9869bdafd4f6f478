"""Compressed branch + top-n in the NSA paper's geometry on the device:
overlapping windows (32 tokens at stride 16) as compressed keys, BS-64
selection scores aggregated from the window scores, block 0 and the two
local blocks forced. Not in the reference (parity unpinned): checked against
the CPU restatement (oracle/attention.py), output at rtol = atol = 0.03,
block scores within 1e-4, and the selection bit-exactly against the ordering
rule applied to the kernel's own block scores."""

import pytest
import torch

from cxlsparse_b200 import ops
from cxlsparse_b200.segments import SegmentLayout
from oracle import attention as A

pytestmark = pytest.mark.gpu

L, D = 32, 16


def _run(query, keys, positions, total, bs, forced, segments=None, window=L, stride=D):
    geometry = ops.select_geometry(len(query), query.shape[1], len(keys), total, bs, 16,
                                   segments=segments, window=window, stride=stride,
                                   forced=forced)
    scores = torch.zeros(len(query), query.shape[1], ops.score_columns(geometry),
                         device="cuda")
    out, blocks = ops.compressed_attention_select(
        query.cuda(), keys.cuda(), positions.cuda(), total, bs, 16, scores=scores,
        segments=segments, window=window, stride=stride, forced=forced)
    torch.cuda.synchronize()
    return out.cpu().float(), blocks.cpu().long(), scores.cpu()


@pytest.mark.parametrize("history,extend,forced", [
    (1000, 64, True),      # tcgen05 kernel
    (16384, 256, True),    # H16K/E256 headline shape (1039 keys)
    (16384, 256, False),
    (40000, 32, True),     # more than 2048 keys: score rows in the global scratch
])
def test_nsa_geometry_matches_oracle(cuda, history, extend, forced):
    bs = 64
    g = torch.Generator().manual_seed(history + extend)
    rows = min(extend, 64)
    positions = torch.arange(history + extend - rows, history + extend, dtype=torch.int32)
    total = history + extend
    keys = torch.randn((total - L) // D + 1, 2, 128, generator=g).bfloat16()
    query = torch.randn(rows, 2, 16, 64, generator=g).bfloat16()
    out, blocks, scores = _run(query, keys, positions, total, bs, forced)
    exp_out, exp_blocks, exp_scores = A.compressed_select_nsa(query, keys, positions, total, bs,
                                                              16, L, D, forced)
    torch.testing.assert_close(out, exp_out, rtol=0.03, atol=0.03)
    # Only candidates (blocks before the row's current block) are scored.
    candidate = (torch.arange(scores.shape[-1])[None, None, :]
                 < (positions.long() // bs)[:, None, None])
    torch.testing.assert_close(scores * candidate, exp_scores * candidate, rtol=1e-4, atol=1e-4)
    rule = A.topn_forced(scores, positions, bs, 16, total, forced)
    assert torch.equal(blocks, rule)
    current = positions.long() // bs
    assert (blocks[:, :, 0] == current[:, None]).all()
    if forced:
        assert (blocks[:, :, 1] == current[:, None] - 1).all()
        assert (blocks[:, :, 2] == 0).all()


def test_identity_geometry_with_forced_blocks(cuda):
    """window = stride = block: the reference summaries, plus forced blocks."""
    bs, history, extend = 64, 5000, 100
    g = torch.Generator().manual_seed(7)
    positions = torch.arange(history, history + extend, dtype=torch.int32)
    total = history + extend
    keys = torch.randn(total // bs, 2, 128, generator=g).bfloat16()
    query = torch.randn(extend, 2, 16, 64, generator=g).bfloat16()
    out, blocks, scores = _run(query, keys, positions, total, bs, True, window=bs, stride=bs)
    base_out, base_blocks = ops.compressed_attention_select(
        query.cuda(), keys.cuda(), positions.cuda(), total, bs, 16)
    assert torch.equal(out, base_out.cpu().float())
    assert torch.equal(blocks, A.topn_forced(scores, positions, bs, 16, total, True))


@pytest.mark.parametrize("history,extend,candidates", [
    (1000, 64, 3), (4096, 64, 3),
    (4096, 128, 4),  # H4K, 4 candidates x 128, BS 64 (the CPU-runnable case)
])
def test_nsa_geometry_over_candidate_segments(cuda, history, extend, candidates):
    """Candidate segments with overlapping windows: the key slots of the
    windows that cross the history boundary are per candidate."""
    bs = 64
    layout = SegmentLayout(history, extend, candidates, bs)
    start, tokens = layout.segments()
    seg_key = (start - L) // D + 1
    seg_keys = tokens // D
    g = torch.Generator().manual_seed(history)
    total = layout.total
    true_keys = [torch.randn((total - L) // D + 1, 2, 128, generator=g).bfloat16()
                 for _ in range(candidates)]
    shared = torch.randn(seg_key, 2, 128, generator=g).bfloat16()
    for c in range(candidates):
        true_keys[c][:seg_key] = shared
    buffer = torch.zeros(seg_key + candidates * seg_keys, 2, 128, dtype=torch.bfloat16)
    buffer[:seg_key] = shared
    for c in range(candidates):
        own = true_keys[c][seg_key:]
        buffer[seg_key + c * seg_keys: seg_key + c * seg_keys + len(own)] = own
    rows = candidates * extend
    query = torch.randn(rows, 2, 16, 64, generator=g).bfloat16()
    positions = torch.tensor(layout.positions(), dtype=torch.int32)
    out, blocks, scores = _run(query, buffer, positions, total, bs, True,
                               segments=layout.segments())
    for c in range(candidates):
        rs = slice(c * extend, (c + 1) * extend)
        true_pos = torch.arange(history, history + extend)
        exp_out, _, exp_scores = A.compressed_select_nsa(query[rs], true_keys[c], true_pos,
                                                         total, bs, 16, L, D, True)
        torch.testing.assert_close(out[rs], exp_out, rtol=0.03, atol=0.03)
        # The kernel's scores in true block order, and its picks mapped back.
        cols = [layout.segment_block(c, j) for j in range(exp_scores.shape[-1])]
        mine = scores[rs][:, :, cols]
        visible = torch.arange(exp_scores.shape[-1])[None, None, :] < (true_pos // bs)[:, None, None]
        torch.testing.assert_close(mine * visible, exp_scores * visible, rtol=1e-4, atol=1e-4)
        got = blocks[rs].clone()
        mapped = got.clone()
        for idx, b in enumerate(got.flatten().tolist()):
            if b >= 0:
                mapped.view(-1)[idx] = layout.true_block(b)
                assert layout.candidate_of(b * bs) in (None, c)
        assert torch.equal(mapped, A.topn_forced(mine, true_pos, bs, 16, total, True))
