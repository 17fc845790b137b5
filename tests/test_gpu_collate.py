"""Cross-request collation on the B200 backend.

Requests collated into shared packed batches under a token budget
(crates/huncho-core/src/engine.rs:554-706) answer as each request does alone:
the same choices and probabilities within the batch-invariance gate of
padded_batch.rs:25-83 (1e-4), through `eval_collated` directly and through
the `BatchQueue` worker thread (batch.rs:85-193) over a two-replica pool.
"""
import pytest

pytestmark = pytest.mark.gpu

from huncho_b200 import collate, engine, synth
from huncho_b200.replicas import ReplicaPool


def _requests(wl):
    by = {}
    for r, p, t, k in zip(wl.rows, wl.positions, wl.qtypes, wl.request_of):
        q = (engine.Question("noul") if t == "noul" else
             engine.Question("choice", labels=[f"L{i}" for i in range(len(p))]) if t == "choice" else
             engine.Question("score", descriptions=[f"level {i}" for i in range(len(p))]))
        req = by.setdefault(k, collate.ScoringRequest([], [], []))
        req.rows.append([int(x) for x in r])
        req.positions.append([int(x) for x in p])
        req.questions.append(q)
    return [by[k] for k in sorted(by)]


def _close(a, b, tol=1e-4):
    assert a["type"] == b["type"]
    assert a.get("choice") == b.get("choice")
    for key in ("noul", "score", "confidence"):
        if key in b:
            assert abs(a[key] - b[key]) <= tol, (key, a[key], b[key])
    for lab, v in b.get("probabilities", {}).items():
        assert abs(a["probabilities"][lab] - v) <= tol


@pytest.fixture(scope="module")
def mini(native_lib, synth_root):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from huncho_b200.backend import KevBackend
    d = synth.write_model(synth_root / "kev-mini-bf16", name="kev-mini", seed=0, store="bf16")
    return KevBackend(d, device=0, dtype="bf16", max_context=4096)


def test_collated_requests_answer_as_alone(mini):
    wl = synth.make_workload(2, mini.vocab_size, seed=9, n_requests=12)
    reqs = _requests(wl)
    stats = collate.EvalStats()
    got = collate.eval_collated(mini, reqs, 2048, stats=stats)
    assert stats.forward_calls > 1 and stats.cross_request_batches >= 1
    assert stats.processed_tokens == wl.n_tokens and stats.padded_tokens == 0
    for req, resp in zip(reqs, got):
        alone = engine.score_questions(mini, req.rows, req.positions, req.questions)
        assert resp.prompt_tokens == sum(len(r) for r in req.rows)
        for a, b in zip(resp.answers, alone):
            _close(a, b)


def test_batch_queue_on_replicas(mini):
    wl = synth.make_workload(2, mini.vocab_size, seed=10, n_requests=10)
    reqs = _requests(wl)
    pool = ReplicaPool([mini, mini.replica()])
    with collate.BatchQueue(pool, capacity=32, max_requests=4, wait_ms=50, tokens=4096) as q:
        futs = [q.submit(r) for r in reqs]
        got = [f.result(timeout=120) for f in futs]
    assert sum(q.group_sizes) == len(reqs) and max(q.group_sizes) <= 4
    for req, resp in zip(reqs, got):
        alone = engine.score_questions(mini, req.rows, req.positions, req.questions)
        for a, b in zip(resp.answers, alone):
            _close(a, b)
