"""Generate golden fixtures by running the reference implementation itself.

Usage:  python tests/golden/make_golden.py <reference project root>

The reference (Sispheqgj/cxlsparse) is Python. This script imports it from the
given checkout and runs:

* ``ActivePlanAdapter.plan`` / ``QueryPrivatePlanAdapter.plan``
  (``cxl_recsys/models/nsa/planning/{active,query_private}.py``) through the
  Triton CPU interpreter (``TRITON_INTERPRET=1``) on CPU tensors, for several
  residency modes, block sizes and read orders;
* ``ops.compressed_attention_select`` / ``ops.window_attention`` torch CPU paths
  (``cxl_recsys/models/nsa/ops.py``);
* ``backends/io_plan.py:selected_attention_oracle`` (FP64);
* the independent dense backbone oracle ``dense_oracle``
  (``tests/test_nsa.py:152-236``) on CPU.

Outputs are small ``.npz`` files beside this script. The tests read only those
files; nothing at test time needs the reference checkout.
"""

import os
import sys
from pathlib import Path
from types import SimpleNamespace

import numpy as np

HERE = Path(__file__).resolve().parent


def _setup(reference_root):
    os.environ["TRITON_INTERPRET"] = "1"
    sys.path.insert(0, str(reference_root))


def _cache(rows, hot, max_history, dim=128):
    import torch

    return SimpleNamespace(
        hot=hot,
        pool=None,
        tags=torch.full((rows, hot + 1), -1, dtype=torch.int32),
        locs=torch.arange(rows * (hot + 1), dtype=torch.int32).reshape(rows, hot + 1),
        host_locs=torch.full((rows, max_history), -1, dtype=torch.int64),
        data=torch.zeros((rows * (hot + 1), dim), dtype=torch.bfloat16),
        max_history=max_history,
    )


PLAN_KEYS = (
    "active_counts", "active_keys", "required", "stats", "address", "hbm", "slots",
    "valid", "starts", "flags", "region_counts", "all_ids", "all_counts",
    "positions", "ioids", "ranks", "missing", "frequencies",
)


def plan_case(name, *, seed, queries, heads, width, bs, hot, old, current,
              residency, read_order, private=False, regions=1, page_size=64,
              pad_rows=0, map_blocks=None, consumer_ctas=None, max_history=None):
    """One planner fixture from the reference planner under the interpreter."""
    import torch

    from cxl_recsys.models.nsa.planning.active import ActivePlanAdapter
    from cxl_recsys.models.nsa.planning.query_private import QueryPrivatePlanAdapter

    g = torch.Generator().manual_seed(seed)
    total = old + current
    max_history = max_history or (old + 64)
    rows_cache = heads
    cache = _cache(rows_cache, hot, max_history)
    pool_pages = (heads * (old + page_size) // page_size) + 2
    cache.pool = SimpleNamespace(backend="cxl" if regions > 1 else "dram",
                                 region_count=regions, pages=pool_pages,
                                 page_size=page_size)
    # Backing slots: a shuffled page list per head, so pages are not adjacent.
    page_perm = torch.randperm(pool_pages, generator=g)
    pages_per_head = -(-old // page_size)
    for h in range(heads):
        pages = page_perm[h * pages_per_head:(h + 1) * pages_per_head]
        token = torch.arange(old)
        cache.host_locs[h, :old] = pages[token // page_size] * page_size + token % page_size
    # Hot residency per head.
    for h in range(heads):
        if residency == "hit":
            hot_tokens = list(range(min(old, hot)))
        elif residency == "partial":
            pool = torch.randperm(old, generator=g)[: min(hot, old) // 2].tolist()
            hot_tokens = sorted(pool)
        else:
            hot_tokens = []
        if hot_tokens:
            cache.tags[h, : len(hot_tokens)] = torch.tensor(hot_tokens, dtype=torch.int32)
    # Selections: random, with duplicates, causal tails and invalid future picks.
    q_total = queries + pad_rows
    positions = torch.full((q_total,), -1, dtype=torch.int64)
    positions[:queries] = old + torch.arange(queries) % max(current, 1)
    blocks = torch.full((q_total, heads, width), -1, dtype=torch.int32)
    if residency != "empty":
        for q in range(queries):
            current_block = int(positions[q]) // bs
            for h in range(heads):
                picks = torch.randint(0, current_block + 1, (width,), generator=g)
                picks[0] = current_block
                drop = torch.rand(width, generator=g) < 0.15
                picks[drop] = -1
                blocks[q, h] = picks.to(torch.int32)
    current_kv = [torch.zeros((max(current, 1), 128), dtype=torch.bfloat16)
                  for _ in range(heads)]
    fetches = [dict(row=h, cached_length=old, history_length=old,
                    current_kv=current_kv[h][:current]) for h in range(heads)]
    query = torch.zeros((q_total, heads, 16, 64), dtype=torch.bfloat16)
    adapter_cls = QueryPrivatePlanAdapter if private else ActivePlanAdapter
    adapter = adapter_cls(cache, chunk_blocks=64)
    w = adapter.allocate(query, blocks, fetches, bs, map_blocks=map_blocks,
                         occurrence_only=True, read_order=read_order)
    w["consumer_ctas"] = consumer_ctas or min(256, w["rows"])
    current_ptr = [0x7F0000000000 + h * 0x100000 for h in range(heads)]
    desc = torch.tensor([(h, old, old, current_ptr[h], current) for h in range(heads)],
                        dtype=torch.int64)
    bases = torch.tensor([0x500000000000 + r * 0x10000000 for r in range(regions)],
                         dtype=torch.int64)
    chosen = adapter.plan(blocks, positions, desc, bases, w, read_order=read_order)
    out = dict(
        blocks=blocks.numpy(), positions=positions.numpy(), desc=desc.numpy(),
        tags=cache.tags.numpy(), locs=cache.locs.numpy(),
        host_locs=cache.host_locs.numpy(), bases=bases.numpy(),
        hot_data=np.int64(cache.data.data_ptr()),
        bs=bs, hot=hot, map_blocks=w["map_blocks"], pool_tokens=pool_pages * page_size,
        page_size=page_size, consumer_ctas=w["consumer_ctas"],
        read_order=read_order, private=int(private),
        chosen=chosen.numpy(),
    )
    for key in PLAN_KEYS:
        out["ref_" + key] = w[key].numpy()
    if read_order.startswith("consumption_depth"):
        out["ref_first_depth"] = w["dependency_first_depth"].numpy()
        out["ref_near"] = w["dependency_near_consumers"].numpy()
    if private:
        out["ref_hot_canonical"] = w["hot_canonical"].numpy()
        out["ref_private_mapping"] = w["mapping"].numpy()
    np.savez_compressed(HERE / f"plan_{name}.npz", **out)
    return out


def attention_case(seed=71):
    """Selected attention FP64 oracle on the reference transport test geometry."""
    import torch

    from cxl_recsys.models.nsa.backends.io_plan import selected_attention_oracle

    g = torch.Generator().manual_seed(seed)
    backing = torch.randn(80, 2, 128, generator=g).bfloat16()
    query = torch.randn(13, 2, 16, 64, generator=g).bfloat16()
    positions = torch.arange(67, 80)
    blocks = torch.tensor([[[0, 1, 0, 4], [1, 0, 1, 4]]] * 13, dtype=torch.int32)
    blocks[3] = -1
    expected = selected_attention_oracle(query, backing, blocks, positions, 16)
    np.savez_compressed(
        HERE / "attention_selected.npz",
        backing=backing.view(torch.int16).numpy(), query=query.view(torch.int16).numpy(),
        positions=positions.numpy(), blocks=blocks.numpy(), expected=expected.numpy())


def select_cases():
    """Compressed attention + top-n and window attention, torch CPU paths."""
    import torch

    from cxl_recsys.models.nsa import ops

    out = {}
    for i, (length, bs, count, chunk) in enumerate(
            [(300, 16, 16, 40), (4096 + 128, 64, 16, 24), (97, 16, 16, 33)]):
        g = torch.Generator().manual_seed(100 + i)
        blocks_total = length // bs
        key = torch.randn(blocks_total, 2, 64, generator=g).bfloat16()
        value = torch.randn(blocks_total, 2, 64, generator=g).bfloat16()
        query = torch.randn(chunk, 2, 16, 64, generator=g).bfloat16()
        positions = torch.arange(length - chunk, length)
        o, sel = ops.compressed_attention_select(
            query.float(), key.float(), value.float(), positions, length, bs, count)
        out[f"c{i}_query"] = query.view(torch.int16).numpy()
        out[f"c{i}_key"] = key.view(torch.int16).numpy()
        out[f"c{i}_value"] = value.view(torch.int16).numpy()
        out[f"c{i}_positions"] = positions.numpy()
        out[f"c{i}_meta"] = np.array([length, bs, count])
        out[f"c{i}_output"] = o.numpy()
        out[f"c{i}_selected"] = sel.numpy()
    # Deterministic ties (tests/test_nsa_fla.py:39-54): zero scores everywhere.
    q = torch.zeros(3, 2, 16, 64)
    kv = torch.zeros(40, 2, 64)
    pos = torch.tensor([17, 95, 401])
    _, tie = ops.compressed_attention_select(q, kv, kv, pos, 640, 16, 16)
    out["tie_selected"] = tie.numpy()
    out["tie_positions"] = pos.numpy()
    # Window branch CPU path (ops.py:194-205).
    g = torch.Generator().manual_seed(9)
    window, start, extend = 64, 200, 40
    records = torch.randn(window - 1 + extend, 2, 128, generator=g).bfloat16()
    query = torch.randn(extend, 2, 16, 64, generator=g).bfloat16()
    positions = torch.arange(start + window - 1, start + window - 1 + extend)
    local = ops.window_attention(query.float(), records.float(), positions, start,
                                 window, 16)
    out["win_records"] = records.view(torch.int16).numpy()
    out["win_query"] = query.view(torch.int16).numpy()
    out["win_positions"] = positions.numpy()
    out["win_meta"] = np.array([window, start])
    out["win_output"] = local.numpy()
    np.savez_compressed(HERE / "select_window.npz", **out)


DENSE_LENGTHS = (7, 17, 143, 256)


def dense_case(reference_root, seed=2024):
    """Whole-backbone output of the reference's independent dense oracle
    (tests/test_nsa.py:152-236) on a 2-layer model of its test checkpoint's
    geometry (hidden 32, 32 / 2 heads of 64, BS 16, window 128, rope theta
    5e5), random weights (norm gains included), at its test lengths 7 / 17 /
    143 and at the selection limit 256. The oracle is written for "cuda"; it
    runs here on CPU with its module's `torch.tensor` / `torch.arange` device
    argument dropped and `Tensor.cuda` as the identity, nothing else changed.
    Importing the test module pulls in the reference's RPC module, whose
    `orjson` import is satisfied by a JSON stand-in (the oracle never uses it)."""
    import importlib.util
    import json
    import types

    import torch

    sys.modules.setdefault("orjson", types.SimpleNamespace(
        dumps=lambda o, **_: json.dumps(o).encode(), loads=json.loads))
    spec = importlib.util.spec_from_file_location(
        "reference_test_nsa", Path(reference_root) / "tests" / "test_nsa.py")
    module = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(module)

    class _CpuTorch:
        def __getattr__(self, name):
            attr = getattr(torch, name)
            if name in ("tensor", "arange"):
                return lambda *args, device=None, **kw: attr(*args, **kw)
            return attr

    module.torch = _CpuTorch()
    hidden, inter, vocab, layers = 32, 64, 256, 2
    g = torch.Generator().manual_seed(seed)

    def normal(*shape, scale=0.2, mean=0.0):
        return (torch.randn(shape, generator=g) * scale + mean).bfloat16()

    weights = {"model.embed_tokens.weight": normal(vocab, hidden, scale=1.0),
               "model.norm.weight": normal(hidden, scale=0.1, mean=1.0)}
    for layer in range(layers):
        p = f"model.layers.{layer}."
        for name in ("input_layernorm.weight", "post_attention_layernorm.weight"):
            weights[p + name] = normal(hidden, scale=0.1, mean=1.0)
        for name, shape in {"self_attn.q_proj.weight": (2048, hidden),
                            "self_attn.k_proj.weight": (128, hidden),
                            "self_attn.v_proj.weight": (128, hidden),
                            "self_attn.o_proj.weight": (hidden, 2048),
                            "self_attn.g_proj.weight": (96, hidden),
                            "mlp.gate_proj.weight": (inter, hidden),
                            "mlp.up_proj.weight": (inter, hidden),
                            "mlp.down_proj.weight": (hidden, inter)}.items():
            weights[p + name] = normal(*shape)
    cfg = SimpleNamespace(selected_tokens=256, rope_theta=500000.0, rms_norm_eps=1e-5,
                          num_hidden_layers=layers)
    out = {f"w:{k}": v.view(torch.int16).numpy() for k, v in weights.items()}
    cuda = torch.Tensor.cuda
    torch.Tensor.cuda = lambda self, *args, **kw: self
    try:
        for length in DENSE_LENGTHS:
            ids = torch.randint(0, vocab, (length,), generator=g)
            expected = module.dense_oracle(ids.tolist(), cfg, weights)
            out[f"ids_{length}"] = ids.numpy()
            out[f"out_{length}"] = expected.view(torch.int16).numpy()
    finally:
        torch.Tensor.cuda = cuda
    out["meta"] = np.array([layers, 16, 128])  # layers, block size, window
    np.savez_compressed(HERE / "dense_model.npz", **out)


CPU_LAYER = dict(hidden=128, q_heads=8, kv_heads=2, head_dim=64, ffn=192, history=640,
                 extend=40, block_size=64, block_counts=4, window=96, tile=16)


def cpu_layer_case(seed=2025):
    """One NSA extend layer through the reference's own CPU torch route, in
    fp32: ``NSAModel._project`` (RMSNorm, q/k/v/g projections, rotary),
    ``ops.append_compressed``, ``ops.local_branches(..., backend="torch")``
    (compressed branch, top-n, window), ``ops.indexed_attention`` over the
    selected tokens packed per KV head as the model's ``selected_finish``
    packs them, and ``NSAModel._finish`` (gate mix, o_proj, FFN)
    (``models/nsa/model.py:440-492, 828-857``, ``models/nsa/ops.py:12-205``).
    The model methods run on a stand-in ``self`` carrying only the fields
    they read. The CPU baseline restatement (oracle/nsa_cpu.py) is pinned to
    this output."""
    import json
    import types

    import torch

    # The model module's import chain reaches the RPC module, whose `orjson`
    # import a JSON stand-in satisfies (nothing here uses it).
    sys.modules.setdefault("orjson", types.SimpleNamespace(
        dumps=lambda o, **_: json.dumps(o).encode(), loads=json.loads))
    from cxl_recsys.models.nsa import ops
    from cxl_recsys.models.nsa.model import NSAModel

    c = CPU_LAYER
    hidden, q_heads, kv_heads, d, ffn = (c[k] for k in ("hidden", "q_heads", "kv_heads",
                                                         "head_dim", "ffn"))
    history, extend, bs, window = c["history"], c["extend"], c["block_size"], c["window"]
    groups = q_heads // kv_heads
    g = torch.Generator().manual_seed(seed)

    def normal(*shape, scale=0.05):
        return (torch.randn(shape, generator=g) * scale).bfloat16().float()

    shapes = {"self_attn.q_proj.weight": (q_heads * d, hidden),
              "self_attn.k_proj.weight": (kv_heads * d, hidden),
              "self_attn.v_proj.weight": (kv_heads * d, hidden),
              "self_attn.g_proj.weight": (q_heads * 3, hidden),
              "self_attn.o_proj.weight": (hidden, q_heads * d),
              "mlp.gate_proj.weight": (ffn, hidden), "mlp.up_proj.weight": (ffn, hidden),
              "mlp.down_proj.weight": (hidden, ffn)}
    weights = {f"model.layers.0.{k}": normal(*s) for k, s in shapes.items()}
    for name in ("input_layernorm.weight", "post_attention_layernorm.weight"):
        weights[f"model.layers.0.{name}"] = torch.ones(hidden)
    model = SimpleNamespace(
        config=SimpleNamespace(num_attention_heads=q_heads, head_dim=d, rms_norm_eps=1e-6),
        heads=kv_heads, groups=groups, weights=weights,
        inv_freq=1.0 / 10000.0 ** (torch.arange(0, d, 2).float() / d))
    model._finish_prepare = lambda *a, **kw: NSAModel._finish_prepare(model, *a, **kw)
    history_kv = normal(history, kv_heads, 2 * d, scale=1.0)
    x = normal(extend, hidden, scale=1.0)
    positions = torch.arange(history, history + extend)
    query, records, gates = NSAModel._project(model, x, positions, 0)
    summaries = history_kv.reshape(-1, bs, kv_heads, 2 * d).float().mean(1)
    compressed, _ = ops.append_compressed(summaries, history_kv[:0], records, bs)
    retained = history_kv[history - (window - 1):]
    cmp_out, win_out, selected = ops.local_branches(
        query, compressed, torch.cat((retained, records)), positions,
        total=history + extend, window_start=history - (window - 1), block_size=bs,
        block_counts=c["block_counts"], window_size=window, tile=c["tile"], backend="torch")
    sequence = torch.cat((history_kv, records))                       # [T, H, 128]
    total = len(sequence)
    values = sequence.permute(1, 0, 2).reshape(kv_heads * total, 2 * d)
    indices = torch.cat([torch.where(selected[:, h] >= 0, selected[:, h] + h * total, -1)
                         for h in range(kv_heads)])
    packed = torch.cat([query[:, h] for h in range(kv_heads)])
    attended = ops.indexed_attention(packed, values, indices, c["tile"])
    selected_out = attended.view(kv_heads, extend, groups, d).transpose(0, 1)
    (out,) = NSAModel._finish(model, x, selected_out, cmp_out, win_out, gates, 0)
    result = {f"w:{k}": v.bfloat16().view(torch.int16).numpy() for k, v in weights.items()}
    result.update(history_kv=history_kv.bfloat16().view(torch.int16).numpy(),
                  hidden=x.bfloat16().view(torch.int16).numpy(),
                  selected=selected.numpy(), compressed_out=cmp_out.numpy(),
                  window_out=win_out.numpy(), selected_out=selected_out.numpy(),
                  output=out.numpy(), meta=np.array([c[k] for k in CPU_LAYER]))
    np.savez_compressed(HERE / "cpu_layer.npz", **result)


def main():
    if len(sys.argv) < 2:
        raise SystemExit(__doc__)
    _setup(Path(sys.argv[1]).resolve())
    if sys.argv[2:] == ["cpu_layer"]:  # regenerate only this fixture
        cpu_layer_case()
        return
    cpu_layer_case()
    dense_case(Path(sys.argv[1]).resolve())
    common = dict(heads=2, hot=32)
    plan_case("miss_bs16_depth", seed=1, queries=13, width=4, bs=16, old=67,
              current=13, residency="miss", read_order="consumption_depth", **common)
    plan_case("partial_bs16_shared", seed=2, queries=13, width=4, bs=16, old=67,
              current=13, residency="partial", read_order="consumption_depth_shared",
              pad_rows=3, **common)
    plan_case("hit_bs16_physical", seed=3, queries=9, width=5, bs=16, old=80,
              current=9, residency="hit", read_order="physical", **common)
    plan_case("empty_bs16", seed=4, queries=5, width=4, bs=16, old=40, current=5,
              residency="empty", read_order="consumption_depth", **common)
    plan_case("partial_bs64_depth", seed=5, queries=48, width=8, bs=64, old=1000,
              current=48, residency="partial", read_order="consumption_depth",
              regions=3, consumer_ctas=7, heads=2, hot=64)
    plan_case("miss_bs64_shared_regions", seed=6, queries=40, width=16, bs=64,
              old=2048, current=40, residency="miss",
              read_order="consumption_depth_shared", regions=2, heads=2, hot=128)
    plan_case("private_partial_bs16", seed=7, queries=13, width=4, bs=16, old=67,
              current=13, residency="partial", read_order="consumption_depth",
              private=True, map_blocks=64, **common)
    plan_case("private_miss_bs64", seed=8, queries=24, width=8, bs=64, old=900,
              current=24, residency="miss", read_order="consumption_depth",
              private=True, regions=2, heads=2, hot=64)
    attention_case()
    select_cases()
    print("fixtures written to", HERE)


if __name__ == "__main__":
    main()
