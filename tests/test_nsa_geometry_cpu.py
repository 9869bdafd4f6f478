"""CPU properties of the NSA-geometry oracle (oracle/attention.py:
compress_mlp, block_scores, topn_forced, compressed_select_nsa), the
restatement that the device's overlapping-window selection is checked
against. Its degenerate case (window = stride = selection block, nothing
forced) is pinned to the reference's own compressed-attention selection on
the golden fixtures; the aggregation weights and forced picks are checked
against the published rule."""

import pytest
import torch

from golden_io import GOLDEN, load
from oracle import attention as A


def _bf(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def test_window_equal_to_block_is_the_reference_selection():
    """l = d = bs, forced off: the same blocks (bit-exact) and output as the
    reference's ops.compressed_attention_select on every golden case."""
    z = load(GOLDEN / "select_window.npz")
    for i in range(3):
        length, bs, count = (int(v) for v in z[f"c{i}_meta"])
        keys = torch.cat((_bf(z[f"c{i}_key"]), _bf(z[f"c{i}_value"])), -1)
        out, selected, scores = A.compressed_select_nsa(
            _bf(z[f"c{i}_query"]).float(), keys, torch.from_numpy(z[f"c{i}_positions"]),
            length, bs, count, bs, bs, False)
        assert torch.equal(selected, torch.from_numpy(z[f"c{i}_selected"]))
        torch.testing.assert_close(out, torch.from_numpy(z[f"c{i}_output"]),
                                   rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("l,d,bs", [(32, 16, 64), (32, 16, 32), (64, 32, 64), (16, 16, 64)])
def test_aggregation_weights_conserve_each_windows_score(l, d, bs):
    """Every window [i d, i d + l) lying inside the scored range spreads its
    score over the blocks it covers with weights summing to l / d (its
    stride steps); for 32 / 16 / 64 an interior block's weights over windows
    4j - 1 .. 4j + 3 are 1, 2, 2, 2, 1."""
    blocks, c = 12, 0
    while c * d + l <= blocks * bs:
        c += 1
    for i in range(c):
        onehot = torch.zeros(1, c, dtype=torch.float64)
        onehot[0, i] = 1.0
        spread = A.block_scores(onehot, l, d, bs, blocks)
        assert spread.sum().item() == l // d, i
        assert (spread >= 0).all()
    if (l, d, bs) == (32, 16, 64):
        j = 5
        weights = [A.overlap_weight(i, j, l, d, bs) for i in range(4 * j - 2, 4 * j + 5)]
        assert weights == [0, 1, 2, 2, 2, 1, 0]


def test_forced_picks_come_first_without_duplicates():
    """Current block, then the previous block and block 0 (when they exist
    and differ), then the rest by score descending with ties to the lower id."""
    scores = torch.zeros(4, 1, 10)
    scores[:, 0, 3], scores[:, 0, 5] = 0.9, 0.9  # a tie: 3 before 5
    positions = torch.tensor([5, 70, 130, 600])  # current blocks 0, 1, 2, 9 at bs 64
    got = A.topn_forced(scores, positions, 64, 5, 640, True)
    assert got[0, 0].tolist() == [0, -1, -1, -1, -1]
    assert got[1, 0].tolist() == [1, 0, -1, -1, -1]
    assert got[2, 0].tolist() == [2, 1, 0, -1, -1]
    assert got[3, 0].tolist() == [9, 8, 0, 3, 5]
    plain = A.topn_forced(scores, positions, 64, 5, 640, False)
    assert plain[3, 0].tolist() == [9, 3, 5, 0, 1]
    assert torch.equal(plain, A.topn_from_scores(scores, positions, 64, 5, 640))


def test_compressed_keys_see_only_complete_windows():
    """A row at position p attends to window i iff i d + l <= p + 1; a row
    before the first complete window attends to nothing (zero output)."""
    torch.manual_seed(0)
    l, d, bs = 32, 16, 64
    keys = torch.randn(10, 1, 128).bfloat16()
    query = torch.randn(3, 1, 16, 64)
    positions = torch.tensor([30, 31, 100])
    out, _, scores = A.compressed_select_nsa(query, keys, positions, 200, bs, 4, l, d, True)
    assert torch.count_nonzero(out[0]) == 0 and torch.count_nonzero(scores[0]) == 0
    torch.testing.assert_close(out[1, 0], keys[0, 0, 64:].float().expand(16, 64))
    # Position 31 sees window 0 alone: block 0 gets weight 2 x 16 heads.
    assert scores[1, 0, 0].item() == pytest.approx(32.0)
    # Position 100 sees windows 0..4, each spread with total weight l / d = 2,
    # so the 16 heads' probabilities (1 each) aggregate to 32 over the blocks.
    assert [i for i in range(10) if i * d + l <= 101] == [0, 1, 2, 3, 4]
    assert scores[2].sum().item() == pytest.approx(32.0, rel=1e-5)
