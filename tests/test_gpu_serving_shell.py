"""The serving shell on the GPU: GR visits through the scheduler and the
worker give what the model gives when called directly.

Two users with 1000-token histories make three visits each; every visit
after the first appends 64 tokens to the user's history (the append-only
prefix of a returning user) and brings a fresh 64-token candidate suffix
with 8 items. The worker prefills only the appended tokens and replays a
captured extend graph. A second model with the same weights, prefilled with
the same history in the same increments, run through its fused extend path
directly, must give the same option logits bit for bit (the same
arithmetic on the same KV values; only the hot-set tiers may differ, and
tiers do not change values). The reference's full-stack check is
tests/test_nsa.py:259-331 (packed append, cold reuse, candidate output).
"""

import pytest
import torch

from cxlsparse_b200.model import NSAConfig, NSAExtendModel
from cxlsparse_b200.serving import ExtendRunner, Scheduler, Worker, gr_sequence

pytestmark = pytest.mark.gpu


def _model(cuda, users):
    return NSAExtendModel(NSAConfig(layers=2, hot=64), device=cuda, seed=0, max_users=users,
                          max_history=1300, chunk=512, workspaces=8)


def test_worker_serves_gr_visits_like_the_model(cuda):
    requests = gr_sequence(2, 1000, 64, warmup=1, measured=2, candidates=8, vocab=32000,
                           seed=5, revisit_tokens=64)
    worker = Worker(ExtendRunner(_model(cuda, 2)), queue_capacity=1)
    try:
        summary = Scheduler(worker).run_sequence(requests, timeout=300)
        assert summary["passed"], summary["worker"]["error"]
        assert summary["worker"]["users"] == {"user-0": {"kv_length": 1128},
                                              "user-1": {"kv_length": 1128}}
    finally:
        worker.close()
    direct = _model(cuda, 2)
    try:
        done = {}
        for request, result in zip(requests, summary["requests"]):
            user, history = request["user_id"], request["history_token_ids"]
            new = history[done.get(user, 0):]
            if new:
                direct.prefill(torch.tensor(new, device=cuda), user=user)
                done[user] = len(history)
            direct.prepare_fast(64, user=user)
            out = direct.extend_fast(torch.tensor(request["candidate_token_ids"],
                                                  device=cuda), user=user)
            logits = (direct.embed[:8].float() @ out[-1].float()).cpu()
            got = result["result"]
            assert got["option_logits"] == [float(v) for v in logits], request["request_id"]
            assert got["recommended_item_id"] == request["candidate_item_ids"][int(logits.argmax())]
            assert got["prompt"]["history_tokens"] == len(history)
            assert got["cache"]["read_bytes"] == got["cache"]["misses"] * 256
            assert result["e2e_ms"] >= result["execution_ms"] > 0
    finally:
        direct.close()


def test_diverging_history_fails_the_worker(cuda):
    requests = gr_sequence(1, 200, 32, warmup=0, measured=2, candidates=4, seed=6)
    requests[1]["history_token_ids"][5] += 1  # no longer extends the cached prefix
    worker = Worker(ExtendRunner(_model(cuda, 1)), queue_capacity=0)
    try:
        summary = Scheduler(worker).run_sequence(requests, timeout=300)
        assert summary["state"] == "FAILED"
        assert "diverges from its cached prefix" in summary["requests"][1]["error"]
    finally:
        worker.close()
