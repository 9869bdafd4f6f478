"""NSA-shaped model glue: chunked prefill into the pool, eager vs graph extend."""

import pytest
import torch

from cxlsparse_b200.model import NSAConfig, NSAExtendModel

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("compression,length", [("mean", 2048), ("mlp", 2048), ("mlp", 2000)])
def test_prefill_then_extend_graph_matches_eager(cuda, compression, length):
    cfg = (NSAConfig(layers=2, hot=64) if compression == "mean"
           else NSAConfig.baseline(layers=2, hot=64))
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_history=length + 64, chunk=512,
                           hot_policy="static")
    try:
        g = torch.Generator().manual_seed(3)
        history = torch.randint(0, cfg.vocab, (length,), generator=g).to(cuda)
        ids = torch.randint(0, cfg.vocab, (64,), generator=g).to(cuda)
        model.prefill(history)
        st = model.user("user")
        assert st.length == length
        assert model.pool.write_bytes == length * cfg.layers * cfg.kv_heads * 256
        # The pool holds exactly the records the cache slot table points at.
        assert (model.cache.host_locs[: cfg.layers * cfg.kv_heads, :length] >= 0).all()
        if compression == "mlp":  # one key per complete 32-token window at stride 16
            assert all(len(k) == (length - 32) // 16 + 1 for k in st.summaries)
        eager = model.extend(ids).clone()
        model.prepare_fast(64)
        fast = model.extend_fast(ids).clone()
        torch.testing.assert_close(fast.float(), eager.float(), rtol=0.02, atol=0.02)
        graph, static_ids, static_out, counters = model.capture_extend(64)
        static_ids.copy_(ids)
        graph.replay()
        torch.cuda.synchronize()
        assert torch.isfinite(static_out).all()
        torch.testing.assert_close(static_out.float(), eager.float(), rtol=0.02, atol=0.02)
        rows = [c.materialize() for c in counters]
        assert len(rows) == cfg.layers
        assert sum(r[0]["misses"] + r[1]["misses"] for r in rows) > 0
    finally:
        model.close()


def test_mlp_compression_matches_oracle(cuda):
    """The model's window compressor (bf16 GEMMs) against the fp32 CPU
    restatement of the NSA compression MLP."""
    from oracle import attention as A

    cfg = NSAConfig.baseline(layers=1)
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_history=512)
    try:
        w = model.layers[0]
        g = torch.Generator().manual_seed(9)
        records = torch.randn(200, 2, 128, generator=g).bfloat16()
        windows = records.unfold(0, 32, 16).permute(0, 3, 1, 2).contiguous()
        got = model.compress(w, windows.cuda()).float().cpu()
        weights = {f"{part}_{name}": w[f"cmp_{name}"][i].cpu()
                   for i, part in enumerate("kv") for name in ("pe", "w1", "w2")}
        expected = A.compress_mlp(records, weights, 32, 16).float()
        assert got.shape == expected.shape == ((200 - 32) // 16 + 1, 2, 128)
        torch.testing.assert_close(got, expected, rtol=0.02, atol=0.01)
    finally:
        model.close()
