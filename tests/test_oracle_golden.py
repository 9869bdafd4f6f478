"""The CPU oracle against fixtures produced by running the reference itself.

Fixtures come from tests/golden/make_golden.py: the reference planner
(planning/active.py, planning/query_private.py) executed through the Triton
CPU interpreter, and the reference's torch NSA ops / FP64 oracles.
"""

import numpy as np
import pytest
import torch

from golden_io import EXACT_KEYS, GOLDEN, load, oracle_args, plan_fixtures
from oracle import attention as A
from oracle import plan as P


@pytest.mark.parametrize("path", plan_fixtures(), ids=lambda p: p.stem)
def test_plan_oracle_matches_reference_planner(path):
    z = load(path)
    fn = P.private_plan if int(z["private"]) else P.active_plan
    out = fn(**oracle_args(z))
    for key in EXACT_KEYS:
        assert np.array_equal(np.asarray(out[key], np.int64), z["ref_" + key].astype(np.int64)), key
    for h, count in enumerate(out["active_counts"]):
        assert np.array_equal(out["active_keys"][h, :count], z["ref_active_keys"][h, :count])
    missing = int(out["missing"])
    assert missing == int(z["ref_missing"][0])
    assert np.array_equal(out["ioids"][:missing], z["ref_ioids"][:missing])
    flags = out["flags"].astype(bool)
    if str(z["read_order"]) != "physical":
        assert np.array_equal(out["ranks"][flags], z["ref_ranks"][flags])
        assert np.array_equal(out["first_depth"][flags], z["ref_first_depth"][flags])
    hot = int(z["hot"])
    assert np.array_equal(out["chosen"][:, :hot], z["chosen"][:, :hot])
    if int(z["private"]):
        assert np.array_equal(out["canonical"], z["ref_hot_canonical"])
        assert np.array_equal(out["private_mapping"], z["ref_private_mapping"])


def _bf(a):
    return torch.from_numpy(a).view(torch.bfloat16)


def test_selection_and_window_oracles_match_reference_ops():
    z = load(GOLDEN / "select_window.npz")
    for i in range(3):
        length, bs, count = (int(v) for v in z[f"c{i}_meta"])
        out, selected, _ = A.compressed_attention_select(
            _bf(z[f"c{i}_query"]).float(), _bf(z[f"c{i}_key"]).float(),
            _bf(z[f"c{i}_value"]).float(), torch.from_numpy(z[f"c{i}_positions"]),
            length, bs, count)
        assert torch.equal(selected, torch.from_numpy(z[f"c{i}_selected"]))
        assert torch.equal(out, torch.from_numpy(z[f"c{i}_output"]))
    window, start = (int(v) for v in z["win_meta"])
    local = A.window_attention(_bf(z["win_query"]).float(), _bf(z["win_records"]).float(),
                               torch.from_numpy(z["win_positions"]), start, window)
    torch.testing.assert_close(local, torch.from_numpy(z["win_output"]), rtol=1e-6, atol=1e-6)


def test_tie_rule_known_answer():
    """Zero scores: [current] + range(min(current, 15)) (tests/test_nsa_fla.py:39-54)."""
    q = torch.zeros(3, 2, 16, 64)
    kv = torch.zeros(40, 2, 64)
    positions = torch.tensor([17, 95, 401])
    _, blocks, _ = A.compressed_attention_select(q, kv, kv, positions, 640, 16, 16)
    for row, p in enumerate((17, 95, 401)):
        current = p // 16
        expected = [current] + list(range(min(current, 15)))
        expected += [-1] * (16 - len(expected))
        assert blocks[row, 0].tolist() == expected
        assert torch.equal(blocks[row, 0], blocks[row, 1])
    z = load(GOLDEN / "select_window.npz")
    assert torch.equal(blocks, torch.from_numpy(z["tie_selected"]))


def test_future_summaries_are_invisible():
    """Selection ignores summaries after the query (tests/test_nsa_ops.py:98-114)."""
    torch.manual_seed(70)
    key = torch.randn(45, 2, 64)
    value = torch.randn_like(key)
    query = torch.randn(3, 2, 16, 64)
    pos = torch.tensor([17, 95, 401])
    first, blocks, _ = A.compressed_attention_select(query, key, value, pos, 720, 16, 16)
    key[26:] = 1e4
    value[26:] = 1e4
    second, other, _ = A.compressed_attention_select(query, key, value, pos, 720, 16, 16)
    assert torch.equal(first, second) and torch.equal(blocks, other)


def test_selected_attention_oracle_matches_reference_fp64():
    z = load(GOLDEN / "attention_selected.npz")
    out = A.selected_attention(_bf(z["query"]), _bf(z["backing"]),
                               torch.from_numpy(z["blocks"]), torch.from_numpy(z["positions"]), 16)
    assert torch.equal(out, torch.from_numpy(z["expected"]))


def test_append_compressed_boundaries():
    """Summary boundaries and an ephemeral suffix (tests/test_nsa_ops.py:10-26)."""
    torch.manual_seed(6)
    values = torch.randn(199, 2, 128).bfloat16()
    compressed, tail, start = values[:0], values[:0], 0
    for stop in (1, 15, 16, 17, 31, 32, 65, 129, 199):
        compressed, tail = A.append_compressed(compressed, tail, values[start:stop], 16)
        expected = values[: stop // 16 * 16].reshape(-1, 16, 2, 128).float().mean(1).bfloat16()
        assert torch.equal(compressed, expected)
        assert torch.equal(tail, values[stop // 16 * 16: stop])
        start = stop


@pytest.mark.parametrize("length", [7, 17, 143, 256])
def test_dense_oracle_matches_reference_dense_oracle(length):
    """oracle/nsa_dense.py is bit-identical to the reference's independent
    dense backbone oracle (tests/test_nsa.py:152-236, run on CPU by the
    fixture script) on a 2-layer model of its test geometry."""
    from oracle.nsa_dense import dense_forward

    z = load(GOLDEN / "dense_model.npz")
    layers_n, block_size, window = (int(v) for v in z["meta"])
    w = {k[2:]: torch.from_numpy(v).view(torch.bfloat16) for k, v in z.items()
         if k.startswith("w:")}
    names = dict(q="self_attn.q_proj", k="self_attn.k_proj", v="self_attn.v_proj",
                 g="self_attn.g_proj", o="self_attn.o_proj", gate="mlp.gate_proj",
                 up="mlp.up_proj", down="mlp.down_proj", in_norm="input_layernorm",
                 post_norm="post_attention_layernorm")
    layers = [{ours: w[f"model.layers.{i}.{theirs}.weight"] for ours, theirs in names.items()}
              for i in range(layers_n)]
    got = dense_forward(torch.from_numpy(z[f"ids_{length}"]), w["model.embed_tokens.weight"],
                        layers, w["model.norm.weight"], q_heads=32, kv_heads=2, head_dim=64,
                        block_size=block_size, window=window, rope_theta=500000.0, eps=1e-5)
    assert torch.equal(got, torch.from_numpy(z[f"out_{length}"]).view(torch.bfloat16))
