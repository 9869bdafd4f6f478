"""The CPU baseline restatement (oracle/nsa_cpu.py) against the reference's own
CPU torch path for one NSA extend layer.

tests/golden/cpu_layer.npz comes from running the reference itself
(``NSAModel._project``, ``ops.append_compressed``,
``ops.local_branches(..., backend="torch")``, ``ops.indexed_attention`` and
``NSAModel._finish``; see ``cpu_layer_case`` in tests/golden/make_golden.py)
on seeded inputs. The restatement must give the same layer output within
fp32 rounding, and the same selected tokens exactly. This is what makes the
timed CPU baseline (``kind: port``) the reference's arithmetic.
"""

import torch

from golden_io import GOLDEN, load
from oracle.nsa_cpu import CPUExtendPath, compressed_select

NAMES = dict(q="self_attn.q_proj", k="self_attn.k_proj", v="self_attn.v_proj",
             g="self_attn.g_proj", o="self_attn.o_proj", gate="mlp.gate_proj",
             up="mlp.up_proj", down="mlp.down_proj")
META = ("hidden", "q_heads", "kv_heads", "head_dim", "ffn", "history", "extend",
        "block_size", "block_counts", "window", "tile")


def _bf(a):
    return torch.from_numpy(a).view(torch.bfloat16).float()


def _path(z):
    m = dict(zip(META, (int(v) for v in z["meta"])))
    path = CPUExtendPath(layers=1, hidden=m["hidden"], q_heads=m["q_heads"],
                         kv_heads=m["kv_heads"], head_dim=m["head_dim"], ffn=m["ffn"],
                         history=m["history"], block_size=m["block_size"],
                         block_counts=m["block_counts"], window=m["window"])
    path.weights[0] = {ours: _bf(z[f"w:model.layers.0.{theirs}.weight"])
                       for ours, theirs in NAMES.items()}
    kv = _bf(z["history_kv"])
    path.kv[0] = kv
    path.summaries[0] = kv.reshape(-1, m["block_size"], m["kv_heads"], 2 * m["head_dim"]).mean(1)
    return path, m


def test_cpu_port_layer_matches_reference_torch_path():
    z = load(GOLDEN / "cpu_layer.npz")
    path, m = _path(z)
    positions = torch.arange(m["history"], m["history"] + m["extend"])
    with torch.inference_mode():
        out = path.layer(0, _bf(z["hidden"]), positions)
    torch.testing.assert_close(out, torch.from_numpy(z["output"]), rtol=1e-5, atol=1e-5)


def test_cpu_port_selection_matches_reference_tokens():
    """The port's top-n blocks, expanded to tokens, are the reference's."""
    z = load(GOLDEN / "cpu_layer.npz")
    path, m = _path(z)
    bs, heads, d = m["block_size"], m["kv_heads"], m["head_dim"]
    positions = torch.arange(m["history"], m["history"] + m["extend"])
    # Recompute the port's query and summaries exactly as its layer() does.
    from oracle.nsa_cpu import rms_norm, rotary

    w, x = path.weights[0], _bf(z["hidden"])
    h = rms_norm(x, path.norm)
    q = (h @ w["q"].T).view(len(x), m["q_heads"], d)
    k = (h @ w["k"].T).view(len(x), heads, d)
    v = (h @ w["v"].T).view(len(x), heads, d)
    q, k = rotary(q, k, positions, path.inv_freq)
    current = torch.cat((k, v), -1)
    total = m["history"] + m["extend"]
    complete = total // bs
    summaries = torch.cat((path.summaries[0], current[: complete * bs - m["history"]].reshape(
        -1, bs, heads, 2 * d).mean(1)))
    _, selected = compressed_select(q.view(len(x), heads, -1, d), summaries[..., :d],
                                    summaries[..., d:], positions, total, bs,
                                    m["block_counts"])
    tokens = (selected[..., None] * bs + torch.arange(bs)).flatten(-2)
    tokens = tokens.masked_fill((tokens < 0) | (tokens > positions[:, None, None]), -1)
    assert torch.equal(tokens, torch.from_numpy(z["selected"]))
