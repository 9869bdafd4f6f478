"""Every layer's hidden output against a float64 oracle, at the benchmark's shapes.

The model runs its real extend path: chunked prefill into the pinned host
pool, the frequency hot set, the compressed branch and top-n on the device,
the deduplicating fetch plan, host -> HBM fetches of the cold blocks and the
fused window / selected attention with the gate mix, then o_proj and the
FFN. For each layer, oracle/nsa_layer.py recomputes the layer in float64 from
the device's own input to that layer, the history K/V read back from the
pool and the device's block selections for that layer (the selections are
checked bit-exactly elsewhere, on the device's own scores; taking them here
keeps near-ties from choosing different blocks on the two sides). The
reference's full-model check is tests/test_nsa.py:152-254.

Bar (the north star's): per layer and per row, max-abs difference <= 2e-2
and cosine >= 0.9995. The layer's own contribution (output minus input) is
also compared, since the residual stream dominates the output.
"""

import ctypes

import pytest
import torch
import torch.nn.functional as F

from cxlsparse_b200.model import NSAConfig, NSAExtendModel
from oracle.nsa_layer import extend_layer, layer_agreement

pytestmark = pytest.mark.gpu

WEIGHTS = ("q", "k", "v", "g", "o", "gate", "up", "down", "in_norm", "post_norm",
           "cmp_pe", "cmp_w1", "cmp_w2")


def pool_history(model, user, layer):
    """History K || V [old, H, 128] of one layer, read back from the host pool."""
    st, pool = model.users[user], model.pool
    old = st.length
    out = torch.empty(old, model.kv_local, 128, dtype=torch.bfloat16)
    regions = [torch.frombuffer((ctypes.c_uint8 * nbytes).from_address(base),
                                dtype=torch.bfloat16).view(-1, 128)
               for base, nbytes in pool._bases]
    for h in range(model.kv_local):
        slots = torch.tensor(pool.token_slots(st.pages[layer][h], 0, old))
        page = slots // pool.page_size
        region = page % pool.regions
        local = (page // pool.regions) * pool.page_size + slots % pool.page_size
        for r, tokens in enumerate(regions):
            rows = (region == r).nonzero().flatten()
            out[rows, h] = tokens[local[rows]]
    return out


CASES = [
    # history, extend, candidates, compression, layers
    (4096, 128, 1, "mean", 16),
    (16384, 256, 1, "mean", 16),
    (16384, 256, 1, "mlp", 16),
    (4096, 256, 3, "mean", 16),
    (16384, 128, 3, "mlp", 4),
]


@pytest.mark.parametrize("history,extend,candidates,compression,layers", CASES,
                         ids=lambda v: str(v))
def test_each_layer_matches_float64_oracle(cuda, history, extend, candidates, compression,
                                           layers):
    cfg = (NSAConfig(layers=layers) if compression == "mean"
           else NSAConfig.baseline(layers=layers))
    model = NSAExtendModel(cfg, device=cuda, seed=history + candidates,
                           max_history=history + candidates * extend + 64 * candidates,
                           workspaces=layers + 4)
    try:
        g = torch.Generator().manual_seed(history * 7 + extend)
        model.prefill(torch.randint(0, cfg.vocab, (history,), generator=g).to(cuda))
        ids = torch.randint(0, cfg.vocab, (candidates * extend,), generator=g).to(cuda)
        model.prepare_fast(extend, candidates=candidates)
        model.extend_fast(ids)  # steady state: the hot set of a previous step is committed
        torch.cuda.synchronize()
        model.counters.clear()
        model.selections, model.layer_outputs = [], []
        inputs = F.embedding(ids, model.embed)
        model.extend_fast(ids)
        torch.cuda.synchronize()
        stats = torch.stack([c.statistics for c in model.counters]).cpu()
        assert int(stats[..., 3].sum()) > 0, "no cold block was fetched"
        assert not stats[..., 6].any() and not any(int(c.device_error.item())
                                                   for c in model.counters)
        layout = model.fast["layout"]
        positions = torch.arange(history, history + extend, device=cuda)
        geometry = dict(q_heads=cfg.q_heads, kv_heads=cfg.kv_heads, head_dim=cfg.head_dim,
                        block_size=cfg.block_size, window=cfg.window,
                        rope_theta=cfg.rope_theta, eps=cfg.rms_eps,
                        compression=cfg.compression, cmp_block=cfg.cmp_block,
                        cmp_stride=cfg.cmp_stride)
        worst = []
        for layer in range(layers):
            weights = {k: v for k, v in model.layers[layer].items() if k in WEIGHTS}
            history_kv = pool_history(model, "user", layer).to(cuda)
            blocks = model.selections[layer].long()
            if candidates > 1:  # segment block ids -> true block ids
                mapped = torch.tensor([layout.true_block(b) for b in blocks.flatten().tolist()],
                                      device=cuda).view_as(blocks)
                blocks = torch.where(blocks >= 0, mapped, blocks)
            layer_in = inputs if layer == 0 else model.layer_outputs[layer - 1]
            got = model.layer_outputs[layer]
            for c in range(candidates):
                rows = slice(c * extend, (c + 1) * extend)
                want = extend_layer(layer_in[rows], weights, history_kv, positions,
                                    blocks[rows], **geometry)
                diff, cos = layer_agreement(got[rows], want)
                _, delta_cos = layer_agreement(got[rows].double() - layer_in[rows].double(),
                                               want - layer_in[rows].double())
                worst.append((layer, c, diff, cos, delta_cos))
        print("\nlayer parity (layer, candidate, max-abs, min cosine, min delta cosine):")
        print("worst max-abs", max(worst, key=lambda t: t[2]))
        print("worst cosine", min(worst, key=lambda t: t[3]))
        print("worst delta cosine", min(worst, key=lambda t: t[4]))
        for layer, c, diff, cos, delta_cos in worst:
            assert diff <= 2e-2 and cos >= 0.9995, (layer, c, diff, cos)
            assert delta_cos >= 0.999, (layer, c, delta_cos)
    finally:
        model.close()
