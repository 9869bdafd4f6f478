"""Several users served by one model on one GPU (the multi-user serving shape,
scaled down): jittered history lengths with partial tail blocks, one captured
extend graph per user, replayed one after another on one stream."""

import pytest
import torch

from cxlsparse_b200.model import NSAConfig, NSAExtendModel

pytestmark = pytest.mark.gpu


def test_users_replayed_back_to_back_match_their_eager_extends(cuda):
    cfg = NSAConfig(layers=2, hot=64)
    histories = {"u0": 1000, "u1": 1337, "u2": 777}  # none a multiple of 64
    extend = 64
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_users=len(histories),
                           max_history=max(histories.values()) + extend, chunk=512,
                           workspaces=cfg.layers * len(histories) + 4)
    try:
        g = torch.Generator().manual_seed(11)
        ids = {}
        for user, length in histories.items():
            model.prefill(torch.randint(0, cfg.vocab, (length,), generator=g).to(cuda), user=user)
            ids[user] = torch.randint(0, cfg.vocab, (extend,), generator=g).to(cuda)
        rows = {u: model.user(u).row for u in histories}
        assert len(set(rows.values())) == len(rows)
        eager = {u: model.extend(ids[u], user=u).clone() for u in histories}
        graphs = {}
        for user in histories:
            graph, static_ids, static_out, counters = model.capture_extend(extend, user=user)
            static_ids.copy_(ids[user])
            graphs[user] = (graph, static_out, counters, static_ids)
        assert all(w.get("pinned") for k, w in model.transport.workspaces.items()
                   if k[-1] is not None)
        for _ in range(2):  # back to back, twice: no user disturbs another
            for user in histories:
                graphs[user][0].replay()
            torch.cuda.synchronize()
            for user in histories:
                out = graphs[user][1]
                torch.testing.assert_close(out.float(), eager[user].float(), rtol=0.02,
                                           atol=0.02)
        for user in histories:
            counts = [c.materialize() for c in graphs[user][2]]
            # Partial tail blocks are fetched through the token gather path.
            assert sum(r[0]["misses"] + r[1]["misses"] for r in counts) > 0
    finally:
        model.close()


def test_users_with_candidate_segments_replay_back_to_back(cuda):
    """configs[3] with candidate segments: each user's request holds 2
    candidates over that user's own jittered history; every user's captured
    graph, replayed back to back with the others, reproduces that user's
    eager segmented step bit for bit."""
    cfg = NSAConfig(layers=2, hot=64)
    histories = {"u0": 1000, "u1": 1337, "u2": 777}
    extend, candidates = 64, 2
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_users=len(histories),
                           max_history=max(histories.values()) + extend + 64, chunk=512,
                           workspaces=cfg.layers * len(histories) + 4)
    try:
        g = torch.Generator().manual_seed(12)
        ids = {}
        for user, length in histories.items():
            model.prefill(torch.randint(0, cfg.vocab, (length,), generator=g).to(cuda), user=user)
            ids[user] = torch.randint(0, cfg.vocab, (candidates * extend,), generator=g).to(cuda)
        eager = {}
        for user in histories:
            model.prepare_fast(extend, user, candidates)
            eager[user] = model.extend_fast(ids[user]).clone()
            torch.cuda.synchronize()
            model.counters.clear()
        graphs = {}
        for user in histories:
            graph, static_ids, static_out, counters = model.capture_extend(
                extend, user=user, candidates=candidates)
            static_ids.copy_(ids[user])
            graphs[user] = (graph, static_out, counters, static_ids)
        for _ in range(2):
            for user in histories:
                graphs[user][0].replay()
            torch.cuda.synchronize()
            for user in histories:
                assert torch.equal(graphs[user][1], eager[user]), user
        for user in histories:
            assert sum(r["misses"] for c in graphs[user][2] for r in c.materialize()) > 0
    finally:
        model.close()


def test_users_with_own_workspaces_replay_concurrently_on_two_streams(cuda):
    """With per-user workspaces the captured graphs of different users share
    no buffer, so they run at the same time on two streams (one user's fetch
    under another's compute). Three users with two candidate segments each,
    users alternating over the two streams, three rounds: every replay still
    reproduces that user's eager step bit for bit."""
    cfg = NSAConfig(layers=2, hot=64)
    histories = {"u0": 1000, "u1": 1337, "u2": 777}
    extend, candidates = 64, 2
    model = NSAExtendModel(cfg, device=cuda, seed=0, max_users=len(histories),
                           max_history=max(histories.values()) + extend + 64, chunk=512,
                           workspaces=cfg.layers * len(histories) + 4, user_workspaces=True)
    try:
        g = torch.Generator().manual_seed(13)
        ids = {}
        for user, length in histories.items():
            model.prefill(torch.randint(0, cfg.vocab, (length,), generator=g).to(cuda), user=user)
            ids[user] = torch.randint(0, cfg.vocab, (candidates * extend,), generator=g).to(cuda)
        eager = {}
        for user in histories:
            model.prepare_fast(extend, user, candidates)
            eager[user] = model.extend_fast(ids[user]).clone()
            torch.cuda.synchronize()
            model.counters.clear()
        graphs = {}
        for user in histories:
            graph, static_ids, static_out, counters = model.capture_extend(
                extend, user=user, candidates=candidates)
            static_ids.copy_(ids[user])
            graphs[user] = (graph, static_out, counters, static_ids)
        pinned = [k for k, w in model.transport.workspaces.items() if w.get("pinned")]
        assert sorted(k[-1] for k in pinned) == sorted(
            (u, i) for u in histories for i in range(cfg.layers))
        main = torch.cuda.current_stream(cuda)
        lanes = [torch.cuda.Stream(cuda) for _ in range(2)]
        for _ in range(3):
            for lane in lanes:
                lane.wait_stream(main)
            for i, user in enumerate(histories):
                with torch.cuda.stream(lanes[i % 2]):
                    graphs[user][0].replay()
            for lane in lanes:
                main.wait_stream(lane)
            torch.cuda.synchronize()
            for user in histories:
                assert torch.equal(graphs[user][1], eager[user]), user
        for user in histories:
            counts = [r for c in graphs[user][2] for r in c.materialize()]
            assert sum(r["misses"] for r in counts) > 0
    finally:
        model.close()
