"""Cross-request collation (huncho_b200.collate) on the CPU.

* `padded_groups` against the cases the reference's own grouping tests check
  (crates/huncho-core/src/engine/batching.rs:83-190): rectangles within the
  budget and padding percentage, caller order kept, no input dropped or
  truncated, 129 one-token rows in groups of 64, 64, 1, prefix contexts
  charged in the workspace but not in the padding bound, readout limits;
* `packed_groups`: the packed-varlen budget (logical tokens) and the same
  order, row and readout rules;
* `eval_collated` against each request evaluated alone (answers, usage,
  batch and cross-request counters), group-wide failure, validation;
* `BatchQueue` (batch.rs:85-193): groups of at most `max_requests`, the
  waiting window from the first request's enqueue time, cancelled requests
  skipped, one backend failure failing its whole group only, a full or closed
  queue answering Unavailable, a closed pool failing the worker.
A fake backend stands in for the GPU: its logits depend only on the row, as
the B200 backend's packed rows do.
"""
import threading
import time

import numpy as np
import pytest

from huncho_b200 import calibration, collate, engine
from huncho_b200.backend import BatchLimits, ForwardInput
from huncho_b200.errors import BackendError, RequestError, UnavailableError, WorkerFailedError
from huncho_b200.replicas import ReplicaPool

F32 = np.float32


class FakeBackend:
    """Host stand-in for KevBackend.score_answers: per-row logits from the
    row's own tokens, host calibration, and device-style answer records."""
    max_context = 4096
    temperature = 1.7

    def __init__(self, fail_token=None, delay=0.0):
        self.calls = []
        self.fail_token = fail_token
        self.delay = delay

    def batch_limits(self):
        return BatchLimits()

    def score_answers(self, tokens, cu, pos, cup, qtypes, temperature=None):
        t = self.temperature if temperature is None else temperature
        n_rows = len(cu) - 1
        assert len(qtypes) == n_rows
        self.calls.append([int(cu[i + 1] - cu[i]) for i in range(n_rows)])
        if self.delay:
            time.sleep(self.delay)
        probs, recs = [], []
        for i in range(n_rows):
            row = np.asarray(tokens[cu[i]:cu[i + 1]], np.int64)
            if self.fail_token is not None and self.fail_token in row:
                raise BackendError("backend failed on a row")
            ps = pos[cup[i]:cup[i + 1]]
            logits = np.array([3.0 * np.sin(0.37 * row[p] + 0.011 * (int(row.sum()) % 97) + 0.1 * p)
                               for p in ps], F32)
            p = calibration.calibrate(logits, t)
            best = calibration.argmax(p.tolist())
            qt = qtypes[i]
            conf = calibration.confidence_score(p) if qt == "score" else calibration.confidence_peak(p)
            if qt == "noul":
                value = float(p[1])
            elif qt == "score":
                value = float(sum(np.float32(j) * p[j] for j in range(len(p))))
            else:
                value = float(p[best])
            probs.append(p)
            recs.append((best, 0, conf, value))
        rec = np.array(recs, dtype=[("best", np.int32), ("status", np.int32), ("confidence", np.float32),
                                    ("value", np.float32)])
        return (np.concatenate(probs) if probs else np.zeros(0, F32)), rec


def _request(rng, n_questions, vocab=1000):
    rows, positions, questions = [], [], []
    for _ in range(n_questions):
        kind = rng.choice(["choice", "noul", "score"])
        n_opt = 2 if kind == "noul" else int(rng.integers(2, 6))
        length = int(rng.integers(n_opt + 2, 200))
        rows.append(rng.integers(0, vocab, length).tolist())
        positions.append(sorted(rng.choice(np.arange(length - 1), n_opt, replace=False).tolist()))
        if kind == "choice":
            questions.append(engine.Question("choice", labels=[f"c{j}" for j in range(n_opt)]))
        elif kind == "score":
            questions.append(engine.Question("score", descriptions=[f"s{j}" for j in range(n_opt)]))
        else:
            questions.append(engine.Question("noul"))
    return collate.ScoringRequest(rows, positions, questions)


def _inputs(lengths, positions=None):
    return [(i, ForwardInput(tokens=[1] * n, positions=positions(n) if positions else [n - 1]))
            for i, n in enumerate(lengths)]


# ------------------------------------------------------------------ grouping
def test_padded_groups_bound_rectangles_padding_and_rows():
    lengths = [1, 2, 3, 3, 4, 5, 7, 9, 10, 35, 80]
    for percent in (0, 1, 25, 100):
        groups = collate.padded_groups(_inputs(lengths), 64, percent, BatchLimits())
        seen = []
        for g in groups:
            rect = len(g) * max(len(x.tokens) for _, x in g)
            logical = sum(len(x.tokens) for _, x in g)
            assert len(g) <= 64
            if len(g) > 1:
                assert rect <= 64
                assert (rect - logical) * 100 <= rect * percent
            for i, x in g:
                assert len(x.tokens) == lengths[i] and list(x.positions) == [lengths[i] - 1]
                seen.append(i)
        assert seen == list(range(len(lengths)))  # caller order, nothing dropped; 80 runs alone
    many = _inputs([1] * 129)
    assert [len(g) for g in collate.padded_groups(many, 4096, 25, BatchLimits())] == [64, 64, 1]


def test_padded_groups_prefix_charges_workspace_not_padding():
    two = _inputs([10, 20], positions=lambda n: [0])
    # 10 padded positions over 40 submitted ones exceeds 24 %, although over
    # the whole 240-token workspace it would look cheap.
    assert len(collate.padded_groups(two, 240, 24, BatchLimits(), prefix=100)) == 2
    assert len(collate.padded_groups(two, 240, 25, BatchLimits(), prefix=100)) == 1
    assert len(collate.padded_groups(two, 239, 25, BatchLimits(), prefix=100)) == 2


def test_groups_split_on_readout_and_row_limits_without_dropping():
    limits = BatchLimits(max_rows=4, max_readouts=256)
    for fn in (lambda x: collate.padded_groups(x, 8192, 0, limits), lambda x: collate.packed_groups(x, 8192, limits)):
        groups = fn(_inputs([256] * 7, positions=lambda n: [3] * 99))
        assert [len(g) for g in groups] == [2, 2, 2, 1]
        assert [i for g in groups for i, _ in g] == list(range(7))
        assert [len(g) for g in fn(_inputs([3] * 3, positions=lambda n: [1] * 300))] == [1, 1, 1]


def test_packed_groups_charge_logical_tokens():
    lengths = [1, 2, 3, 3, 4, 5, 7, 9, 10, 35, 80]
    groups = collate.packed_groups(_inputs(lengths), 64, BatchLimits())
    assert [i for g in groups for i, _ in g] == list(range(len(lengths)))
    for g in groups:
        if len(g) > 1:
            assert sum(len(x.tokens) for _, x in g) <= 64
    # packed rows carry no padding, so fewer batches than exact-length rectangles
    assert len(groups) < len(collate.padded_groups(_inputs(lengths), 64, 0, BatchLimits()))
    assert [len(g) for g in groups] == [9, 1, 1]  # 1+2+...+10 = 44 tokens; 44+35 and 35+80 exceed 64


# ---------------------------------------------------------------- collation
def _alone(backend, req):
    """The request evaluated by itself, one row per call."""
    out = []
    for r, p, q in zip(req.rows, req.positions, req.questions):
        out += collate.eval_batched(backend, [r], [p], [q], 1 << 30)
    return out


def _same_answers(a, b):
    assert a["type"] == b["type"]
    for key in ("choice", "noul", "score", "confidence"):
        assert a.get(key) == b.get(key)
    assert a.get("probabilities") == b.get("probabilities")


@pytest.mark.parametrize("packed,percent", [(True, 0), (False, 0), (False, 50), (False, 100)])
def test_eval_collated_equals_requests_alone(packed, percent):
    rng = np.random.default_rng(4)
    reqs = [_request(rng, int(rng.integers(1, 6))) for _ in range(9)]
    b = FakeBackend()
    stats = collate.EvalStats()
    got = collate.eval_collated(b, reqs, 700, percent=percent, packed=packed, stats=stats)
    assert len(got) == len(reqs)
    for req, resp in zip(reqs, got):
        assert resp.prompt_tokens == sum(len(r) for r in req.rows)
        alone = _alone(FakeBackend(), req)
        assert len(resp.answers) == len(alone)
        for x, y in zip(resp.answers, alone):
            _same_answers(x, y)
        for q, a in zip(req.questions, resp.answers):
            assert a["type"] == q.type
    n_rows = sum(len(r.rows) for r in reqs)
    assert sum(len(c) for c in b.calls) == n_rows
    assert stats.forward_calls == len(b.calls)
    assert stats.batch_calls == sum(len(c) > 1 for c in b.calls)
    for c in b.calls:  # every native batch within the budget (or a lone oversized row)
        cost = sum(c) if packed else max(c) * len(c)
        assert len(c) == 1 or cost <= 700
        assert c == sorted(c)  # rows enter by length
    if packed:
        assert stats.processed_tokens == sum(len(r) for q in reqs for r in q.rows) and stats.padded_tokens == 0
        assert stats.cross_request_batches >= 1
    else:
        assert stats.processed_tokens == sum(max(c) * len(c) for c in b.calls)
        assert stats.padded_tokens == sum(max(c) * len(c) - sum(c) for c in b.calls)
        if percent == 0:
            assert stats.padded_tokens == 0 and all(len(set(c)) == 1 for c in b.calls)


def test_eval_collated_host_answers_match_engine():
    """The scattered answers are Engine::build_answer's for the same probabilities."""
    rng = np.random.default_rng(8)
    req = _request(rng, 6)
    b = FakeBackend()
    [resp] = collate.eval_collated(b, [req], 4096)
    for r, p, q, a in zip(req.rows, req.positions, req.questions, resp.answers):
        probs, _ = FakeBackend().score_answers(np.asarray(r, np.uint32), np.array([0, len(r)]), np.asarray(p),
                                               np.array([0, len(p)]), [q.type])
        h = engine.build_answer(q, engine.candidates_for(q, p), probs)
        for key in ("choice", "type"):
            assert a.get(key) == h.get(key)
        for key in ("noul", "score", "confidence"):
            if key in h:
                assert abs(a[key] - h[key]) <= 1e-6


def test_eval_collated_validation_and_group_failure():
    rng = np.random.default_rng(1)
    reqs = [_request(rng, 2) for _ in range(3)]
    b = FakeBackend()
    with pytest.raises(RequestError):
        collate.eval_collated(b, [], 100)
    with pytest.raises(RequestError):
        collate.eval_collated(b, reqs * 22, 100)  # 66 requests
    with pytest.raises(RequestError):
        collate.eval_collated(b, reqs, 0)
    with pytest.raises(RequestError):
        collate.eval_batched(b, reqs[0].rows, reqs[0].positions, reqs[0].questions, 100, percent=101)
    cached = collate.ScoringRequest(reqs[0].rows, reqs[0].positions, reqs[0].questions, prefix_cache=True)
    with pytest.raises(RequestError):
        collate.eval_collated(b, [reqs[1], cached], 100)
    with pytest.raises(RequestError):
        collate.eval_collated(b, [collate.ScoringRequest(reqs[0].rows, reqs[0].positions[:1], reqs[0].questions)], 100)
    long = collate.ScoringRequest([[1] * 5000], [[3, 4]], [engine.Question("noul")])
    with pytest.raises(RequestError):
        collate.eval_collated(b, [reqs[0], long], 1 << 20)
    assert not b.calls  # every check runs before any backend work
    poisoned = collate.ScoringRequest([[7, 7, 999_999, 7]], [[0, 1]], [engine.Question("noul")])
    with pytest.raises(BackendError):
        collate.eval_collated(FakeBackend(fail_token=999_999), reqs + [poisoned], 1 << 20)


# --------------------------------------------------------------- batch queue
def _pool(*backends):
    return ReplicaPool(list(backends) or [FakeBackend()])


def test_batch_queue_collates_up_to_max_requests():
    rng = np.random.default_rng(2)
    reqs = [_request(rng, 3) for _ in range(10)]
    b = FakeBackend()
    with collate.BatchQueue(_pool(b), capacity=64, max_requests=4, wait_ms=300, tokens=1 << 20) as q:
        futs = [q.submit(r) for r in reqs]
        got = [f.result(timeout=10) for f in futs]
    assert q.group_sizes == [4, 4, 2]
    assert q.stats.cross_request_batches >= 1
    for req, resp in zip(reqs, got):
        for x, y in zip(resp.answers, _alone(FakeBackend(), req)):
            _same_answers(x, y)


def test_batch_queue_window_starts_at_first_enqueue():
    rng = np.random.default_rng(3)
    b = FakeBackend()
    with collate.BatchQueue(_pool(b), capacity=8, max_requests=8, wait_ms=150, tokens=1 << 20) as q:
        t0 = time.monotonic()
        f1 = q.submit(_request(rng, 1))
        time.sleep(0.05)
        f2 = q.submit(_request(rng, 1))  # joins the first request's window
        f1.result(timeout=10)
        f2.result(timeout=10)
        waited = time.monotonic() - t0
        assert 0.14 <= waited < 2.0
        assert q.group_sizes == [2]
        assert max(q.queue_wait_s) < 1.0


def test_batch_queue_skips_cancelled_requests():
    rng = np.random.default_rng(5)
    b = FakeBackend()
    with collate.BatchQueue(_pool(b), capacity=8, max_requests=8, wait_ms=200, tokens=1 << 20) as q:
        futs = [q.submit(_request(rng, 1)) for _ in range(4)]
        assert futs[1].cancel() and futs[3].cancel()
        assert futs[0].result(timeout=10).answers and futs[2].result(timeout=10).answers
    assert q.group_sizes == [2]
    assert sum(len(c) for c in b.calls) == 2


def test_batch_queue_failure_fails_only_its_group():
    rng = np.random.default_rng(6)
    b = FakeBackend(fail_token=999_999)
    poisoned = collate.ScoringRequest([[5, 999_999, 5]], [[0, 1]], [engine.Question("noul")])
    with collate.BatchQueue(_pool(b), capacity=16, max_requests=2, wait_ms=100, tokens=1 << 20) as q:
        futs = [q.submit(r) for r in (_request(rng, 2), poisoned, _request(rng, 2), _request(rng, 2))]
        for f in futs[:2]:
            with pytest.raises(BackendError):
                f.result(timeout=10)
        assert all(f.result(timeout=10).answers for f in futs[2:])

    def boom(backend, requests, budget):
        raise ZeroDivisionError("bug")

    with collate.BatchQueue(_pool(), capacity=4, max_requests=2, wait_ms=10, tokens=100, evaluate=boom) as q:
        with pytest.raises(WorkerFailedError):
            q.submit(_request(rng, 1)).result(timeout=10)


def test_batch_queue_full_closed_and_pool_closed():
    rng = np.random.default_rng(7)
    gate, started = threading.Event(), threading.Event()

    def slow(backend, requests, budget):
        started.set()
        gate.wait(10)
        return [collate.ScoringResponse([], 0) for _ in requests]

    q = collate.BatchQueue(_pool(), capacity=1, max_requests=1, wait_ms=0, tokens=100, evaluate=slow)
    first = q.submit(_request(rng, 1))
    assert started.wait(10)  # the worker holds the first request
    second = q.submit(_request(rng, 1))  # fills the queue
    third = q.submit(_request(rng, 1))
    with pytest.raises(UnavailableError):
        third.result(timeout=1)
    gate.set()
    assert first.result(timeout=10).prompt_tokens == 0 and second.result(timeout=10) is not None
    q.close()
    with pytest.raises(UnavailableError):
        q.submit(_request(rng, 1)).result(timeout=1)

    pool = _pool()
    pool.close()
    q = collate.BatchQueue(pool, capacity=4, max_requests=2, wait_ms=10, tokens=100)
    with pytest.raises(WorkerFailedError):
        q.submit(_request(rng, 1)).result(timeout=10)
    q._worker.join(10)
    assert not q._worker.is_alive()
    with pytest.raises(UnavailableError):  # the worker stopped: nothing is admitted any more
        q.submit(_request(rng, 1)).result(timeout=1)
    q.close()
    with pytest.raises(RequestError):
        collate.BatchQueue(_pool(), capacity=0, max_requests=1, wait_ms=0, tokens=1)


class BarrierBackend(FakeBackend):
    """A fake whose first call waits for the other handles' first calls: it
    only returns if the handles run concurrently."""

    def __init__(self, barrier, **kw):
        super().__init__(**kw)
        self.barrier = barrier

    def score_answers(self, *a, **kw):
        if not self.calls:
            self.barrier.wait(timeout=10)
        return super().score_answers(*a, **kw)


def test_eval_batched_over_replica_handles_runs_them_concurrently():
    rng = np.random.default_rng(11)
    reqs = [_request(rng, 4) for _ in range(6)]
    barrier = threading.Barrier(3)
    handles = [BarrierBackend(barrier) for _ in range(3)]
    stats = collate.EvalStats()
    got = collate.eval_collated(handles[0], reqs, 300, replicas=handles[1:], stats=stats)
    assert stats.forward_calls >= 3 and all(len(h.calls) >= 1 for h in handles)
    assert sum(len(h.calls) for h in handles) == stats.forward_calls
    one = collate.eval_collated(FakeBackend(), reqs, 300)
    for a, b in zip(got, one):
        assert a.prompt_tokens == b.prompt_tokens
        for x, y in zip(a.answers, b.answers):
            _same_answers(x, y)
    # a failing handle fails the call after the others finish
    poisoned = collate.ScoringRequest([[5, 999_999, 5]], [[0, 1]], [engine.Question("noul")])
    bad = [FakeBackend(fail_token=999_999) for _ in range(2)]
    with pytest.raises(BackendError):
        collate.eval_collated(bad[0], reqs + [poisoned], 300, replicas=bad[1:])
    assert all(h.calls for h in bad)
