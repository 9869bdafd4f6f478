"""Serving shell: a GPU worker over the extend model, a scheduler that replays
GR request sequences, and the request contract between them.

The reference serves generative-recommendation (GR) requests through a
Worker with one GPU executor thread and a bounded task queue
(``cxl_recsys/worker/service.py:20-340``), fed by a Scheduler whose
``run_sequence`` admits a finite, timestamped workload and waits for it
(``cxl_recsys/scheduler/service.py:382-475``). A request carries a user's
full history (an immutable prefix that later visits may only extend) and
the candidate suffix (``cxl_recsys/common/request.py``,
``cxl_recsys/worker/prompt.py``). This module keeps those interfaces: the
method names, the request and reply fields, the statuses (QUEUED, RUNNING,
SUCCEEDED, FAILED, ABORTED, UNKNOWN) and the rejection reasons (busy,
record_capacity, run_failed, epoch_mismatch). Underneath, the worker runs
``ExtendRunner``: each user's history lives in the pinned host pool, is
prefilled once and extended in place when a later visit appends to it, and
every (user, history length, suffix length) gets one captured CUDA graph of
the 16-layer extend, replayed per request.

Everything runs in one process per GPU; the scheduler talks to its worker by
method calls (the reference's gRPC transport is out of scope).
"""

import hashlib
import json
import math
import queue
import threading
import time
import uuid
from array import array
from collections import OrderedDict
from dataclasses import dataclass, field

MAX_CANDIDATES = 128
MAX_CANDIDATE_TOKENS = MAX_CANDIDATES * 256
FINISHED = ("SUCCEEDED", "FAILED", "ABORTED")
REQUEST_FIELDS = {"request_id", "user_id", "history_token_ids", "candidates",
                  "candidate_token_ids", "candidate_item_ids", "timestamp", "visit_index"}


# ---------------------------------------------------------------- contract --
def _name(value, what):
    if not isinstance(value, str) or not 0 < len(value) <= 128:
        raise ValueError(f"{what} must be a nonempty string, max 128 characters")
    return value


def _tokens(value, limit):
    if not isinstance(value, list) or not 0 < len(value) <= limit:
        raise ValueError(f"Token sequence must have 1..{limit} entries")
    if set(map(type, value)) != {int} or min(value) < 0 or max(value) >= 2**31:
        raise ValueError("Token IDs must be nonnegative int32")
    return list(value)


def _items(value, limit):
    if not isinstance(value, list) or not 0 < len(value) <= limit:
        raise ValueError("Invalid candidate count")
    for item in value:
        _name(item, "item_id")
    if len(set(value)) != len(value):
        raise ValueError("Candidate item_id values must be unique")
    return list(value)


def parse_request(value, max_history=16384, max_candidates=MAX_CANDIDATES):
    """Validated copy of one request (the reference's contract: history plus
    either ``candidates`` [{item_id, token_ids}] or a flat
    ``candidate_token_ids`` with ``candidate_item_ids``)."""
    if not isinstance(value, dict):
        raise ValueError("Request must be an object")
    unknown = set(value) - REQUEST_FIELDS
    if unknown:
        raise ValueError(f"Unknown request fields: {sorted(unknown)}")
    out = {"request_id": _name(value.get("request_id"), "request_id"),
           "user_id": _name(value.get("user_id"), "user_id"),
           "history_token_ids": _tokens(value.get("history_token_ids"), max_history)}
    flat = {"candidate_token_ids", "candidate_item_ids"} & set(value)
    if "candidates" in value:
        if flat:
            raise ValueError("candidates cannot be mixed with flat candidate fields")
        candidates = value["candidates"]
        if not isinstance(candidates, list) or not 0 < len(candidates) <= max_candidates:
            raise ValueError("Invalid candidate count")
        parsed = []
        for c in candidates:
            if not isinstance(c, dict) or set(c) != {"item_id", "token_ids"}:
                raise ValueError("Each candidate needs item_id and token_ids")
            parsed.append({"item_id": c["item_id"], "token_ids": _tokens(c["token_ids"], 256)})
        _items([c["item_id"] for c in parsed], max_candidates)
        out["candidates"] = parsed
    else:
        out["candidate_token_ids"] = _tokens(value.get("candidate_token_ids"),
                                             MAX_CANDIDATE_TOKENS)
        out["candidate_item_ids"] = _items(value.get("candidate_item_ids"), max_candidates)
    if "timestamp" in value:
        t = value["timestamp"]
        if type(t) not in (int, float) or not math.isfinite(t) or t < 0:
            raise ValueError("timestamp must be a finite nonnegative number")
        out["timestamp"] = t
    if "visit_index" in value:
        if type(value["visit_index"]) is not int or value["visit_index"] < 0:
            raise ValueError("visit_index must be a nonnegative integer")
        out["visit_index"] = value["visit_index"]
    return out


def parse_batch(value, max_history=16384, max_batch_size=16):
    """A batch task: independent users' requests in a stable order."""
    if (not isinstance(value, dict) or not {"batch_id", "requests"} <= set(value)
            or set(value) - {"batch_id", "requests", "expected_epoch"}):
        raise ValueError("Batch needs batch_id and requests, with optional expected_epoch")
    requests = value["requests"]
    if not isinstance(requests, list) or not 0 < len(requests) <= max_batch_size:
        raise ValueError(f"Batch must contain 1..{max_batch_size} requests")
    parsed = [parse_request(r, max_history) for r in requests]
    for key in ("request_id", "user_id"):
        if len({r[key] for r in parsed}) != len(parsed):
            raise ValueError(f"Batch {key} values must be unique")
    return {"batch_id": _name(value["batch_id"], "batch_id"), "requests": parsed}


def fingerprint(value):
    """Payload digest for duplicate detection: token lists hashed as packed
    int32 bytes (a 16K-token history in microseconds), the rest as JSON."""
    h = hashlib.sha256()
    rest = {}
    for key in sorted(value):
        item = value[key]
        if isinstance(item, list) and item and type(item[0]) is int:
            h.update(key.encode() + b"=" + array("i", item).tobytes())
        else:
            rest[key] = item
    h.update(json.dumps(rest, sort_keys=True, separators=(",", ":")).encode())
    return h.hexdigest()


def candidate_suffix(request):
    """The packed candidate suffix (all candidates, in order) and the item ids."""
    if "candidates" in request:
        tokens = [t for c in request["candidates"] for t in c["token_ids"]]
        return tokens, [c["item_id"] for c in request["candidates"]]
    return list(request["candidate_token_ids"]), list(request["candidate_item_ids"])


# ------------------------------------------------------------------ worker --
@dataclass
class _Task:
    batch_id: str
    payload: dict
    request_ids: list
    status: str = "QUEUED"
    queued_ns: int = 0
    fields: dict = field(default_factory=dict)


@dataclass
class _Record:
    request_id: str
    batch_id: str
    position: int
    fingerprint: str
    status: str = "QUEUED"
    fields: dict = field(default_factory=dict)


class Worker:
    """One GPU executor thread serving batch tasks from a bounded queue.

    ``queue_capacity`` tasks may wait behind the running one. A failed task
    poisons the worker: the partial KV state cannot be rolled back, so queued
    tasks are aborted and every later submission is refused (run_failed).
    Resubmitting an accepted request or batch with the same payload is
    answered as a duplicate; a different payload under the same id is an
    error.
    """

    def __init__(self, runner, queue_capacity=1, max_records=10000, max_batch_size=16):
        if queue_capacity < 0 or max_records <= 0 or max_batch_size <= 0:
            raise ValueError("Invalid Worker capacities")
        self.runner = runner
        self.capacity = queue_capacity + 1
        self.max_records, self.max_batch_size = max_records, max_batch_size
        self.epoch = uuid.uuid4().hex
        self._cond = threading.Condition()
        self._tasks = {}
        self._records = {}
        self._pending = queue.Queue()
        self._inflight = 0
        self._closing = False
        self._failure = None
        self._users = {}
        self._thread = threading.Thread(target=self._serve, name="gpu-executor", daemon=True)
        self._thread.start()

    # -- admission ---------------------------------------------------------
    def _refuse(self, reason):
        return {"accepted": False, "reason": reason, "epoch": self.epoch}

    def submit(self, value):
        """One request as a batch of one (the reference's compatibility path)."""
        request = parse_request(value, self.runner.max_history)
        rid = request["request_id"]
        with self._cond:
            if self._failure is not None:
                return self._refuse("run_failed")
            known = self._records.get(rid)
            if known is not None:
                if known.fingerprint != fingerprint(request):
                    raise ValueError("request_id reused with a different payload")
                return {"accepted": True, "duplicate": True, "epoch": self.epoch,
                        "request_id": rid, "batch_id": known.batch_id}
            reply = self._admit({"batch_id": "single-" + uuid.uuid4().hex,
                                 "requests": [request]})
        if reply["accepted"]:
            reply["request_id"] = rid
        return reply

    def submit_batch(self, value):
        if isinstance(value, dict) and "expected_epoch" in value:
            expected = value["expected_epoch"]
            if not isinstance(expected, str) or not 0 < len(expected) <= 128:
                raise ValueError("expected_epoch must be a nonempty string")
            if expected != self.epoch:  # stale owner: refuse before touching any state
                return self._refuse("epoch_mismatch")
            value = {k: v for k, v in value.items() if k != "expected_epoch"}
        batch = parse_batch(value, self.runner.max_history, self.max_batch_size)
        with self._cond:
            return self._admit(batch)

    def _admit(self, batch):  # under the lock
        bid, requests = batch["batch_id"], batch["requests"]
        if self._failure is not None:
            return self._refuse("run_failed")
        known = self._tasks.get(bid)
        if known is not None:
            if known.payload != batch:
                raise ValueError("batch_id reused with a different payload")
            return {"accepted": True, "duplicate": True, "batch_id": bid, "epoch": self.epoch}
        if any(r["request_id"] in self._records for r in requests):
            raise ValueError("request_id already belongs to an accepted batch")
        if self._closing or self._inflight >= self.capacity:
            return self._refuse("busy")
        if len(self._records) + len(requests) > self.max_records:
            return self._refuse("record_capacity")
        task = _Task(bid, batch, [r["request_id"] for r in requests])
        self._tasks[bid] = task
        for position, r in enumerate(requests):
            self._records[r["request_id"]] = _Record(r["request_id"], bid, position,
                                                     fingerprint(r))
        self._inflight += 1
        task.queued_ns = time.perf_counter_ns()
        self._pending.put(task)
        return {"accepted": True, "duplicate": False, "batch_id": bid, "epoch": self.epoch}

    # -- execution ---------------------------------------------------------
    def _set(self, task, status, **fields):  # under the lock
        task.status = status
        task.fields.update(fields)
        for rid in task.request_ids:
            record = self._records[rid]
            record.status = status
            record.fields.update(fields)
        self._cond.notify_all()

    def _serve(self):
        while True:
            task = self._pending.get()
            if task is None:
                return
            with self._cond:
                started = time.perf_counter_ns()
                self._set(task, "RUNNING", queue_wait_ms=(started - task.queued_ns) / 1e6)
            try:
                results = self.runner.execute(task.payload["requests"])
                if len(results) != len(task.request_ids):
                    raise RuntimeError("runner returned a wrong number of results")
                users = self.runner.snapshot()
                elapsed = (time.perf_counter_ns() - started) / 1e6
            except Exception as exc:  # the KV state is now undefined: stop serving
                error = f"{type(exc).__name__}: {exc}"
                with self._cond:
                    self._failure, self._closing, self._users = error, True, {}
                    spent = (time.perf_counter_ns() - started) / 1e6
                    self._set(task, "FAILED", error=error, elapsed_ms=spent, execution_ms=spent)
                    while True:
                        try:
                            queued = self._pending.get_nowait()
                        except queue.Empty:
                            break
                        if queued is not None:
                            self._set(queued, "ABORTED", error="Worker run failed: " + error)
                    self._inflight = 0
                return
            with self._cond:
                self._set(task, "SUCCEEDED", elapsed_ms=elapsed, execution_ms=elapsed)
                for rid, result in zip(task.request_ids, results):
                    record = self._records[rid]
                    record.fields["result"] = result
                    record.fields["user_state"] = users.get(result.get("user_id"))
                self._users = users
                self._inflight -= 1

    # -- queries -----------------------------------------------------------
    def _reply(self, rid):  # under the lock
        record = self._records.get(rid)
        if record is None:
            return {"epoch": self.epoch, "status": "UNKNOWN", "error": self._failure}
        return {"epoch": self.epoch, "run_failed": self._failure is not None,
                "request_id": rid, "batch_id": record.batch_id,
                "batch_position": record.position, "status": record.status,
                **record.fields}

    def get(self, value):
        with self._cond:
            return self._reply(value["request_id"])

    def get_batch(self, value):
        wait_ms = value.get("wait_ms", 0)
        if type(wait_ms) not in (int, float) or not 0 <= wait_ms <= 1000:
            raise ValueError("wait_ms must be between 0 and 1000")
        bid = value["batch_id"]
        with self._cond:
            task = self._tasks.get(bid)
            if wait_ms and task is not None:
                self._cond.wait_for(lambda: task.status in FINISHED or self._failure is not None
                                    or self._closing, timeout=wait_ms / 1000)
            if task is None:
                return {"epoch": self.epoch, "status": "UNKNOWN", "error": self._failure}
            return {"epoch": self.epoch, "run_failed": self._failure is not None,
                    "batch_id": bid, "status": task.status, "request_ids": list(task.request_ids),
                    **task.fields, "requests": [self._reply(r) for r in task.request_ids]}

    def status(self, _=None):
        with self._cond:
            return {"control_features": {"completion_wait": True, "epoch_guarded_submit": True},
                    "epoch": self.epoch, "outstanding": self._inflight,
                    "capacity": self.capacity, "max_batch_size": self.max_batch_size,
                    "records": len(self._records), "batches": len(self._tasks),
                    "users": dict(self._users), "closing": self._closing,
                    "failed": self._failure is not None, "error": self._failure}

    def close(self):
        with self._cond:
            self._closing = True
            self._cond.notify_all()
            if self._failure is None and self._thread.is_alive():
                self._pending.put(None)
        self._thread.join()
        self.runner.close()


# -------------------------------------------------------------- scheduler --
class Scheduler:
    """Replays a finite, timestamped request sequence through a worker.

    Requests are admitted in order; a request with a ``timestamp`` (seconds
    from the start of the run) waits for its arrival, and a busy worker is
    polled every ``poll_s``. Completion is read back from the worker. The
    end-to-end time of a request runs from its admission to the moment the
    scheduler sees it finished.
    """

    def __init__(self, worker, poll_s=0.0005):
        self.worker, self.poll_s = worker, poll_s

    def run_sequence(self, requests, timeout=300.0, stop_event=None):
        if timeout <= 0:
            raise ValueError("run timeout must be positive")
        started = time.monotonic()
        admitted, finished, cursor, state = {}, {}, 0, None
        while state is None:
            now = time.monotonic() - started
            if self.worker.status()["failed"]:
                state = "FAILED"
            elif stop_event is not None and stop_event.is_set():
                state = "INTERRUPTED"
            elif now >= timeout:
                state = "TIMED_OUT"
            if state is not None:
                break
            while cursor < len(requests) and requests[cursor].get("timestamp", 0) <= now:
                reply = self.worker.submit(requests[cursor])
                if not reply["accepted"]:
                    if reply["reason"] not in ("busy", "run_failed"):
                        raise RuntimeError("Admission rejected: " + reply["reason"])
                    break
                admitted[requests[cursor]["request_id"]] = time.monotonic()
                cursor += 1
            for rid in list(admitted):
                if rid not in finished and self.worker.get({"request_id": rid})["status"] in FINISHED:
                    finished[rid] = time.monotonic()
            if cursor == len(requests) and len(finished) == len(requests):
                state = "COMPLETED"
                break
            time.sleep(self.poll_s)
        results = []
        for index, request in enumerate(requests):
            rid = request["request_id"]
            if index < cursor:
                result = self.worker.get({"request_id": rid})
                if rid in finished:
                    result["e2e_ms"] = (finished[rid] - admitted[rid]) * 1e3
            else:
                result = {"request_id": rid, "status": "NOT_SUBMITTED"}
            for key in ("timestamp", "visit_index"):
                if key in request:
                    result[key] = request[key]
            results.append(result)
        succeeded = sum(r["status"] == "SUCCEEDED" for r in results)
        return {"state": state, "passed": state == "COMPLETED" and succeeded == len(requests),
                "total": len(requests), "submitted": cursor, "succeeded": succeeded,
                "elapsed_seconds": time.monotonic() - started, "requests": results,
                "worker": self.worker.status()}


def percentile(values, q):
    """Linear-interpolated percentile (q in [0, 100]) of a nonempty list."""
    ordered = sorted(values)
    if not ordered:
        raise ValueError("no values")
    k = (len(ordered) - 1) * q / 100
    lo = int(math.floor(k))
    hi = min(lo + 1, len(ordered) - 1)
    return ordered[lo] + (ordered[hi] - ordered[lo]) * (k - lo)


# -------------------------------------------------------- GR replay inputs --
def gr_sequence(users, history, extend, *, warmup=3, measured=15, candidates=8, vocab=32000,
                seed=0, revisit_tokens=0):
    """Synthetic GR visits: each user's history (``history`` seeded random
    tokens), then ``warmup + measured`` visits, each with a fresh candidate
    suffix of ``extend`` tokens (``candidates`` items). With
    ``revisit_tokens`` > 0 every visit first appends that many tokens to the
    user's history (the append-only prefix of a returning user). Visits are
    interleaved across users in order; ``visit_index`` counts per user."""
    import random

    rng = random.Random(seed)
    if extend < candidates:
        raise ValueError("extend must hold at least one token per candidate")
    histories = {f"user-{u}": [rng.randrange(vocab) for _ in range(history)]
                 for u in range(users)}
    requests = []
    for visit in range(warmup + measured):
        for user, tokens in histories.items():
            if visit and revisit_tokens:
                tokens.extend(rng.randrange(vocab) for _ in range(revisit_tokens))
            suffix = [rng.randrange(vocab) for _ in range(extend)]
            requests.append({"request_id": f"{user}-visit-{visit}", "user_id": user,
                             "history_token_ids": list(tokens),
                             "candidate_token_ids": suffix,
                             "candidate_item_ids": [f"item-{visit}-{i}"
                                                    for i in range(candidates)],
                             "visit_index": visit})
    return requests


# ------------------------------------------------------------ model runner --
class ExtendRunner:
    """Executes requests on an ``NSAExtendModel``.

    Per user the runner keeps the history tokens it has prefilled into the
    pinned pool; a request's history must start with them (the prefix is
    immutable), and any further tokens are prefilled first. The candidate
    suffix runs as one extend forward (candidates packed into one suffix,
    as the reference packs them, worker/prompt.py:24-55), replayed from a
    CUDA graph captured once per (user, history length, suffix length) and
    kept in an LRU of ``graphs`` entries. Candidate selection scores the
    first len(candidate_item_ids) option tokens (ids 0 .. n - 1, the slots
    of the reference's A-Z option letters) against the final hidden state
    of the suffix's last token with the tied embedding, fp32, and returns
    the argmax item.
    """

    def __init__(self, model, graphs=8):
        self.model = model
        self.max_history = model.max_history
        self.graphs = OrderedDict()
        self.capacity = graphs
        self.histories = {}

    def _prefill(self, user, history):
        import torch

        cached = self.histories.setdefault(user, [])
        if history[:len(cached)] != cached:
            raise ValueError(f"history of {user} diverges from its cached prefix")
        if len(history) > len(cached):
            new = torch.tensor(history[len(cached):], dtype=torch.int64,
                               device=self.model.device)
            self.model.prefill(new, user=user)
            cached.extend(history[len(cached):])
            for key in [k for k in self.graphs if k[0] == user]:
                del self.graphs[key]  # captured against the shorter history

    def _graph(self, user, extend):
        key = (user, len(self.histories[user]), extend)
        if key in self.graphs:
            self.graphs.move_to_end(key)
            return self.graphs[key]
        while len(self.graphs) >= self.capacity:
            self.graphs.popitem(last=False)
        entry = self.model.capture_extend(extend, user=user)
        self.graphs[key] = entry
        return entry

    def execute(self, requests):
        import torch

        results = []
        for request in requests:
            user = request["user_id"]
            history = request["history_token_ids"]
            if len(history) > self.max_history:
                raise ValueError("history exceeds the model's max_history")
            self._prefill(user, history)
            suffix, items = candidate_suffix(request)
            graph, static_ids, static_out, counters = self._graph(user, len(suffix))
            static_ids.copy_(torch.tensor(suffix, dtype=torch.int64), non_blocking=True)
            graph.replay()
            last = static_out[-1].float()
            options = self.model.embed[:len(items)].float()
            logits = (options @ last).cpu()
            stats = torch.stack([c.statistics for c in counters]).cpu()
            choice = int(logits.argmax())
            results.append({
                "request_id": request["request_id"], "user_id": user,
                "postprocessing": "candidate_selection",
                "selected_option": choice, "recommended_item_id": items[choice],
                "option_logits": [float(v) for v in logits],
                "prompt": {"history_tokens": len(history), "candidate_tokens": len(suffix),
                           "input_tokens": len(suffix),
                           "last_input_position": len(history) + len(suffix) - 1},
                "cache": {"hits": int(stats[..., 2].sum()), "misses": int(stats[..., 3].sum()),
                          "read_bytes": int(stats[..., 3].sum()) * 256},
                **{k: request[k] for k in ("timestamp", "visit_index") if k in request}})
        return results

    def snapshot(self):
        return {user: {"kv_length": len(tokens)} for user, tokens in self.histories.items()}

    def close(self):
        self.graphs.clear()
        self.model.close()
