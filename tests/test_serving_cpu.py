"""Serving shell host logic on CPU (cxlsparse_b200/serving.py), with a
stand-in runner: the request contract, worker admission and capacity,
duplicates, epoch guards, failure poisoning, completion waits, and the
scheduler's replay of a timestamped sequence. Restates the reference's
worker and scheduler tests (tests/test_core.py:85-105, 319-356;
tests/test_scheduler.py:53-87, 88-206, 207-258) on this implementation.
"""

import threading
import time

import pytest

from cxlsparse_b200.serving import (Scheduler, Worker, candidate_suffix, gr_sequence,
                                    parse_request, percentile)


def request(rid="r0", user="u0", history=(1, 2, 3), suffix=(7, 8), items=("a", "b"), **extra):
    return {"request_id": rid, "user_id": user, "history_token_ids": list(history),
            "candidate_token_ids": list(suffix), "candidate_item_ids": list(items), **extra}


class FakeRunner:
    """Records calls; optionally blocks until released or fails on a user."""

    max_history = 64

    def __init__(self, gate=None, fail_user=None):
        self.gate, self.fail_user, self.calls, self.closed = gate, fail_user, [], False

    def execute(self, requests):
        if self.gate is not None:
            assert self.gate.wait(5)
        self.calls.append([r["request_id"] for r in requests])
        if any(r["user_id"] == self.fail_user for r in requests):
            raise RuntimeError("device failure")
        return [{"request_id": r["request_id"], "user_id": r["user_id"],
                 "tokens": len(candidate_suffix(r)[0])} for r in requests]

    def snapshot(self):
        return {"u0": {"kv_length": 3}}

    def close(self):
        self.closed = True


def wait_status(worker, rid, status, timeout=5):
    deadline = time.monotonic() + timeout
    while time.monotonic() < deadline:
        if worker.get({"request_id": rid})["status"] == status:
            return
        time.sleep(0.002)
    raise AssertionError(worker.get({"request_id": rid}))


def test_request_contract():
    parsed = parse_request(request(timestamp=1.5, visit_index=2))
    assert parsed["candidate_token_ids"] == [7, 8] and parsed["timestamp"] == 1.5
    packed = parse_request({"request_id": "r", "user_id": "u", "history_token_ids": [1],
                            "candidates": [{"item_id": "x", "token_ids": [4, 5]},
                                           {"item_id": "y", "token_ids": [6]}]})
    assert candidate_suffix(packed) == ([4, 5, 6], ["x", "y"])
    for bad, message in ((request(extra_field=1), "Unknown request fields"),
                         (request(history=()), "Token sequence"),
                         (request(history=(1, -2)), "nonnegative int32"),
                         (request(items=("a", "a")), "unique"),
                         (request(timestamp=-1), "timestamp"),
                         (request(rid=""), "request_id")):
        with pytest.raises(ValueError, match=message):
            parse_request(bad)
    mixed = dict(request(), candidates=[{"item_id": "x", "token_ids": [1]}])
    with pytest.raises(ValueError, match="cannot be mixed"):
        parse_request(mixed)
    with pytest.raises(ValueError, match="Token sequence"):
        parse_request(request(history=range(65)), max_history=64)


def test_worker_capacity_duplicates_and_epoch():
    gate = threading.Event()
    worker = Worker(FakeRunner(gate), queue_capacity=0)
    try:
        first = worker.submit(request("r0"))
        assert first["accepted"] and not first["duplicate"]
        again = worker.submit(request("r0"))
        assert again["accepted"] and again["duplicate"] and again["batch_id"] == first["batch_id"]
        with pytest.raises(ValueError, match="different payload"):
            worker.submit(request("r0", suffix=(9,)))
        assert worker.submit(request("r1", user="u1")) == {
            "accepted": False, "reason": "busy", "epoch": worker.epoch}
        assert worker.submit_batch({"batch_id": "b", "expected_epoch": "stale",
                                    "requests": [request("r2")]})["reason"] == "epoch_mismatch"
        gate.set()
        wait_status(worker, "r0", "SUCCEEDED")
        reply = worker.get({"request_id": "r0"})
        assert reply["result"]["tokens"] == 2 and reply["user_state"] == {"kv_length": 3}
        assert reply["elapsed_ms"] >= 0 and reply["queue_wait_ms"] >= 0
        assert worker.get({"request_id": "nope"})["status"] == "UNKNOWN"
        batch = worker.submit_batch({"batch_id": "b1", "expected_epoch": worker.epoch,
                                     "requests": [request("r3"), request("r4", user="u1")]})
        assert batch["accepted"]
        done = worker.get_batch({"batch_id": "b1", "wait_ms": 1000})
        assert done["status"] == "SUCCEEDED" and [r["status"] for r in done["requests"]] == [
            "SUCCEEDED"] * 2
        with pytest.raises(ValueError, match="unique"):
            worker.submit_batch({"batch_id": "b2", "requests": [request("r5"),
                                                                 request("r6")]})
        status = worker.status()
        assert status["outstanding"] == 0 and status["records"] == 3 and not status["failed"]
    finally:
        gate.set()
        worker.close()


def test_failure_poisons_the_worker_and_aborts_queued_tasks():
    gate = threading.Event()
    runner = FakeRunner(gate, fail_user="bad")
    worker = Worker(runner, queue_capacity=2)
    try:
        assert worker.submit(request("r0", user="bad"))["accepted"]
        assert worker.submit(request("r1"))["accepted"]
        gate.set()
        wait_status(worker, "r0", "FAILED")
        wait_status(worker, "r1", "ABORTED")
        assert "device failure" in worker.get({"request_id": "r0"})["error"]
        assert worker.submit(request("r2"))["reason"] == "run_failed"
        assert worker.status()["failed"] and runner.calls == [["r0"]]
    finally:
        worker.close()
    assert runner.closed


def test_scheduler_replays_a_timestamped_sequence_in_order():
    runner = FakeRunner()
    worker = Worker(runner, queue_capacity=1)
    try:
        requests = [request(f"r{i}", user=f"u{i % 2}", timestamp=0.01 * i) for i in range(6)]
        summary = Scheduler(worker).run_sequence(requests, timeout=30)
        assert summary["state"] == "COMPLETED" and summary["passed"]
        assert [r["request_id"] for r in summary["requests"]] == [f"r{i}" for i in range(6)]
        assert all(r["e2e_ms"] >= 0 and r["timestamp"] == 0.01 * i
                   for i, r in enumerate(summary["requests"]))
        assert [c[0] for c in runner.calls] == [f"r{i}" for i in range(6)]
        assert summary["elapsed_seconds"] >= 0.05  # the last arrival is at 0.05 s
    finally:
        worker.close()


def test_scheduler_stops_on_failure():
    worker = Worker(FakeRunner(fail_user="u1"), queue_capacity=0)
    try:
        summary = Scheduler(worker).run_sequence([request("r0"), request("r1", user="u1"),
                                                  request("r2")], timeout=30)
        assert summary["state"] == "FAILED" and not summary["passed"]
        assert summary["requests"][1]["status"] == "FAILED"
        assert summary["requests"][2]["status"] in ("NOT_SUBMITTED", "ABORTED")
    finally:
        worker.close()


def test_gr_sequence_and_percentile():
    requests = gr_sequence(2, 100, 32, warmup=1, measured=2, candidates=4, revisit_tokens=5)
    assert len(requests) == 6 and requests[0]["user_id"] == "user-0"
    for r in requests:
        parse_request(r, max_history=200)
        assert len(r["candidate_token_ids"]) == 32 and len(r["candidate_item_ids"]) == 4
    first, second = requests[0], requests[2]
    assert second["history_token_ids"][:100] == first["history_token_ids"]
    assert len(second["history_token_ids"]) == 105 and second["visit_index"] == 1
    assert percentile([3, 1, 2], 50) == 2 and percentile([1, 2, 3, 4], 50) == 2.5
