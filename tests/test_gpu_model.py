"""NSA-shaped model glue: chunked prefill into the pool, eager vs graph extend."""

import pytest
import torch

from cxlsparse_b200.model import NSAConfig, NSAExtendModel

pytestmark = pytest.mark.gpu


def test_prefill_then_extend_graph_matches_eager(cuda):
    cfg = NSAConfig(layers=2, hot=64)
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_history=2048 + 64, chunk=512,
                           hot_policy="static")
    try:
        g = torch.Generator().manual_seed(3)
        history = torch.randint(0, cfg.vocab, (2048,), generator=g).to(cuda)
        ids = torch.randint(0, cfg.vocab, (64,), generator=g).to(cuda)
        model.prefill(history)
        st = model.user("user")
        assert st.length == 2048
        assert model.pool.write_bytes == 2048 * cfg.layers * cfg.kv_heads * 256
        # The pool holds exactly the records the cache slot table points at.
        assert (model.cache.host_locs[: cfg.layers * cfg.kv_heads, :2048] >= 0).all()
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
