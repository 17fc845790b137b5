"""Cross-request collation over the B200 Kev backend.

The reference's server gathers concurrent scoring requests into bounded
groups (crates/huncho-api/src/batch.rs:85-193: at most `rows` requests, a
waiting window counted from the first request's enqueue time, callers that
went away skipped before and after a backend is leased). Its engine then runs
the group's question rows as native batches under a token budget and hands
every request its own answers and usage (crates/huncho-core/src/engine.rs:
554-706; eval_batched, engine.rs:1005-1140; grouping, engine/batching.rs:
21-80). A backend failure fails the whole group.

Here each native batch is one `KevBackend.score_answers` call: the rows run
packed back to back, with calibration and answers computed on the device.
Packed rows carry no padding, so `packed_groups` charges a batch its logical
tokens; `padded_groups` keeps the reference's rectangle rule (longest row x
rows, with a padding percentage) for callers that want the reference's exact
batch boundaries. Both keep the caller's order, close a group at
`max_rows`, bound readout rows by `max_readouts`, and run an input that fits
no group alone rather than truncating it.
"""
from __future__ import annotations

import queue
import threading
import time
from concurrent.futures import Future, ThreadPoolExecutor, wait
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

from . import engine
from .backend import BatchLimits, ForwardInput, pack_rows
from .errors import HunchoError, RequestError, UnavailableError, WorkerFailedError

MAX_COLLATED_REQUESTS = 64  # engine.rs:561


@dataclass
class EvalStats:
    """The physical-work counters of EvalStats (engine.rs:76-103) that batching
    moves. `processed_tokens` are the tokens the device ran; `padded_tokens`
    the padding inside them (always 0 for packed batches)."""
    forward_calls: int = 0
    batch_calls: int = 0
    padded_batch_calls: int = 0
    cross_request_batches: int = 0
    processed_tokens: int = 0
    padded_tokens: int = 0

    def accumulate(self, other: "EvalStats") -> None:
        for k in self.__dataclass_fields__:
            setattr(self, k, getattr(self, k) + getattr(other, k))


@dataclass
class ScoringRequest:
    """One request's question rows: token ids, option readout positions and the
    typed question of each row (one Kev question per row)."""
    rows: Sequence[Sequence[int]]
    positions: Sequence[Sequence[int]]
    questions: Sequence[engine.Question]
    prefix_cache: bool = False


@dataclass
class ScoringResponse:
    """The request's answers in question order and its logical token usage."""
    answers: List[dict]
    prompt_tokens: int


def _shape(item):
    inp = item[1]
    return len(inp.tokens), len(inp.positions) + 1  # readout rows: options + decision


def padded_groups(inputs, budget: int, percent: int, limits: Optional[BatchLimits] = None,
                  prefix: int = 0) -> list:
    """Greedy groups of (index, ForwardInput) pairs charging the padded
    rectangle (batching.rs:21-80). A row joins the open group while
    (longest + prefix) x rows <= budget, the readout rows stay within
    `limits.max_readouts`, and the padding (longest x rows minus the rows'
    tokens) is at most `percent` of longest x rows; a group also closes at
    `limits.max_rows` rows."""
    limits = limits or BatchLimits()
    groups, group = [], []
    longest = logical = readouts = 0
    for item in inputs:
        n, cost = _shape(item)
        rows = len(group) + 1
        wide = max(longest, n)
        physical = wide * rows
        new_logical = logical + n
        fits = ((wide + prefix) * rows <= budget
                and (limits.max_readouts is None or readouts + cost <= limits.max_readouts)
                and (physical - new_logical) * 100 <= physical * percent)
        if group and (len(group) == limits.max_rows or not fits):
            groups.append(group)
            group, longest, logical, readouts = [], 0, 0, 0
        longest = max(longest, n)
        logical += n
        readouts += cost
        group.append(item)
    if group:
        groups.append(group)
    return groups


def packed_groups(inputs, budget: int, limits: Optional[BatchLimits] = None, prefix: int = 0) -> list:
    """Greedy groups of (index, ForwardInput) pairs for packed varlen batches:
    a row joins the open group while the rows' tokens plus `prefix` context
    tokens per row stay within `budget` and the readout rows within
    `limits.max_readouts`; a group closes at `limits.max_rows` rows."""
    limits = limits or BatchLimits()
    groups, group = [], []
    logical = readouts = 0
    for item in inputs:
        n, cost = _shape(item)
        rows = len(group) + 1
        fits = (logical + n + prefix * rows <= budget
                and (limits.max_readouts is None or readouts + cost <= limits.max_readouts))
        if group and (len(group) == limits.max_rows or not fits):
            groups.append(group)
            group, logical, readouts = [], 0, 0
        logical += n
        readouts += cost
        group.append(item)
    if group:
        groups.append(group)
    return groups


def eval_batched(backend, rows: Sequence[Sequence[int]], positions: Sequence[Sequence[int]],
                 questions: Sequence[engine.Question], budget: int, *, percent: int = 0, packed: bool = True,
                 origins: Optional[Sequence[int]] = None, temperature: Optional[float] = None,
                 stats: Optional[EvalStats] = None, replicas: Sequence = ()) -> list:
    """Answers of independent question rows run as budgeted native batches
    (engine.rs:1005-1140): rows are ordered by length (stable), grouped, and
    each group is one device call with on-device calibration; answers come
    back in input order. `origins[i]` names the request of row i, so batches
    that mix requests are counted.

    `replicas` are further handles of the same model (`KevBackend.replica()`:
    the package loaded again, own weights, workspace and stream): the batches are dealt to
    `backend` and them round-robin, and each handle's share runs on its own
    host thread (the native call releases the GIL), so batches overlap on the
    GPU. Any batch's failure fails the call, after every thread has ended."""
    if budget <= 0 or not 0 <= percent <= 100:
        raise RequestError("batch token budget must be positive and padding percent 0..100")
    if not (len(rows) == len(positions) == len(questions)):
        raise RequestError("one position list and one question per row are required")
    stats = stats if stats is not None else EvalStats()
    max_context = getattr(backend, "max_context", None)
    for i, r in enumerate(rows):
        if max_context is not None and len(r) > max_context:
            raise RequestError(f"question `{i}` exceeds model input budgets")
    order = sorted(range(len(rows)), key=lambda i: len(rows[i]))
    items = [(i, ForwardInput(tokens=rows[i], positions=positions[i])) for i in order]
    limits = backend.batch_limits()
    groups = (packed_groups(items, budget, limits) if packed
              else padded_groups(items, budget, percent, limits))
    answers: list = [None] * len(rows)
    jobs = []
    for group in groups:
        idx = [i for i, _ in group]
        lengths = [len(rows[i]) for i in idx]
        count = len(idx)
        stats.forward_calls += 1
        if packed:
            stats.processed_tokens += sum(lengths)
        else:
            padding = max(lengths) * count - sum(lengths)
            stats.processed_tokens += max(lengths) * count
            stats.padded_tokens += padding
            stats.padded_batch_calls += int(count > 1 and padding > 0)
        if count > 1:
            stats.batch_calls += 1
            if origins is not None and any(origins[i] != origins[idx[0]] for i in idx):
                stats.cross_request_batches += 1
        jobs.append((idx, [rows[i] for i in idx], [positions[i] for i in idx], [questions[i] for i in idx]))

    handles = [backend, *replicas]
    n_threads = min(len(handles), len(jobs))

    def run(h):
        out = []
        for j in range(h, len(jobs), n_threads):
            idx, rs, ps, qs = jobs[j]
            probs, rec = handles[h].score_answers(*pack_rows(rs, ps), [q.type for q in qs],
                                                  temperature=temperature)
            if len(rec) != len(idx):
                raise HunchoError("batch backend returned the wrong number of sequences")
            out.append((j, probs, rec))
        return out

    if n_threads > 1:
        with ThreadPoolExecutor(max_workers=n_threads) as pool:
            futures = [pool.submit(run, h) for h in range(n_threads)]
            wait(futures)
        results = [x for f in futures for x in f.result()]
    else:
        results = run(0) if jobs else []
    for j, probs, rec in results:
        idx, _, ps, qs = jobs[j]
        k = 0
        for i, q, pos, r in zip(idx, qs, ps, rec):
            n = len(pos)
            answers[i] = engine.answer_from_record(q, engine.candidates_for(q, pos), probs[k:k + n], r)
            k += n
    return answers


def eval_collated(backend, requests: Sequence[ScoringRequest], budget: int, *, percent: int = 0,
                  packed: bool = True, temperature: Optional[float] = None,
                  stats: Optional[EvalStats] = None, replicas: Sequence = ()) -> List[ScoringResponse]:
    """Several requests' questions run as shared native batches, each request
    getting its own answers and usage back (engine.rs:554-706). The whole
    group is checked before any work; a failure of any batch fails the group."""
    if not requests or len(requests) > MAX_COLLATED_REQUESTS or budget <= 0:
        raise RequestError("collation requires 1-64 requests and a positive token budget")
    rows, positions, questions, origins = [], [], [], []
    for k, req in enumerate(requests):
        if req.prefix_cache:
            raise RequestError("collated requests require identical execution options and token budgets "
                               "without prefix reuse")
        if not (len(req.rows) == len(req.positions) == len(req.questions)):
            raise RequestError("one position list and one question per row are required")
        rows.extend(req.rows)
        positions.extend(req.positions)
        questions.extend(req.questions)
        origins.extend([k] * len(req.rows))
    answers = eval_batched(backend, rows, positions, questions, budget, percent=percent, packed=packed,
                           origins=origins, temperature=temperature, stats=stats, replicas=replicas)
    out, s = [], 0
    for req in requests:
        n = len(req.rows)
        out.append(ScoringResponse(answers=answers[s:s + n], prompt_tokens=sum(len(r) for r in req.rows)))
        s += n
    if s != len(answers):
        raise HunchoError("collation omitted a request")
    return out


@dataclass
class _Pending:
    request: ScoringRequest
    future: Future
    queued: float = field(default_factory=time.monotonic)


_STOP = object()


class BatchQueue:
    """Bounded cross-request collation (batch.rs:30-193) on a worker thread.

    `submit` returns a Future at once: it fails with UnavailableError when the
    queue (capacity `capacity`) is full or closed. The worker, started by the
    first submit, takes the oldest request, then collects more until
    `max_requests` are held or `wait_ms` has passed since that first request
    was queued (a late worker does not wait a whole window again), skipping
    cancelled futures; it leases a backend from `pool` (a ReplicaPool),
    skips requests cancelled meanwhile, and runs the group through
    `eval_collated` with the `tokens` budget. A HunchoError from the group
    fails every request in it with that error; any other failure with
    WorkerFailedError. `close` drains what was queued, then stops the worker.
    """

    def __init__(self, pool, capacity: int, max_requests: int, wait_ms: float, tokens: int, *,
                 percent: int = 0, packed: bool = True, temperature: Optional[float] = None,
                 evaluate: Optional[Callable] = None):
        if capacity <= 0 or not 1 <= max_requests <= MAX_COLLATED_REQUESTS or tokens <= 0 or wait_ms < 0:
            raise RequestError("batch queue needs a positive capacity and budget and 1-64 requests per group")
        self._pool = pool
        self._queue: queue.Queue = queue.Queue(maxsize=capacity)
        self._max_requests = max_requests
        self._wait = wait_ms / 1000.0
        self._tokens = tokens
        self.stats = EvalStats()
        self.group_sizes: List[int] = []
        self.queue_wait_s: List[float] = []
        if evaluate is None:
            def evaluate(backend, requests, budget):
                return eval_collated(backend, requests, budget, percent=percent, packed=packed,
                                     temperature=temperature, stats=self.stats)
        self._evaluate = evaluate
        self._lock = threading.Lock()
        self._closed = False
        self._worker: Optional[threading.Thread] = None

    def submit(self, request: ScoringRequest) -> Future:
        fut: Future = Future()
        with self._lock:
            if self._closed:
                fut.set_exception(UnavailableError("batch queue is closed"))
                return fut
            if self._worker is None:
                self._worker = threading.Thread(target=self._run, name="huncho-batch", daemon=True)
                self._worker.start()
            try:
                self._queue.put_nowait(_Pending(request, fut))
            except queue.Full:
                fut.set_exception(UnavailableError("batch queue is full"))
        return fut

    def close(self, timeout: Optional[float] = None) -> None:
        with self._lock:
            if self._closed:
                return
            self._closed = True
            worker = self._worker
        if worker is not None:
            self._queue.put(_STOP)
            worker.join(timeout)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def _run(self) -> None:
        while True:
            first = self._queue.get()
            if first is _STOP:
                return
            if first.future.cancelled():
                continue
            deadline = first.queued + self._wait
            group, stop = [first], False
            while len(group) < self._max_requests:
                try:
                    nxt = self._queue.get_nowait()
                except queue.Empty:
                    remaining = deadline - time.monotonic()
                    if remaining <= 0:
                        break
                    try:
                        nxt = self._queue.get(timeout=remaining)
                    except queue.Empty:
                        break
                if nxt is _STOP:
                    stop = True
                    break
                if not nxt.future.cancelled():
                    group.append(nxt)
            if not self._execute(group) or stop:
                self._fail_queued()
                return

    def _fail_queued(self) -> None:
        with self._lock:
            self._closed = True
        while True:
            try:
                p = self._queue.get_nowait()
            except queue.Empty:
                return
            if p is not _STOP and p.future.set_running_or_notify_cancel():
                p.future.set_exception(WorkerFailedError("batch worker stopped"))

    def _execute(self, group: List[_Pending]) -> bool:
        group = [p for p in group if not p.future.cancelled()]
        if not group:
            return True
        try:
            lease = self._pool.lease()
            backend = lease.__enter__()
        except Exception:  # a closed pool ends the worker; its callers learn it failed
            for p in group:
                if p.future.set_running_or_notify_cancel():
                    p.future.set_exception(WorkerFailedError("no backend available"))
            return False
        try:
            running = [p for p in group if p.future.set_running_or_notify_cancel()]
            if not running:
                return True
            now = time.monotonic()
            self.queue_wait_s.extend(now - p.queued for p in running)
            self.group_sizes.append(len(running))
            try:
                responses = self._evaluate(backend, [p.request for p in running], self._tokens)
            except HunchoError as e:
                for p in running:
                    p.future.set_exception(e)
                return True
            except Exception as e:  # noqa: BLE001 -- any other failure is the worker's
                for p in running:
                    p.future.set_exception(WorkerFailedError(f"batch worker failed: {e!r}"))
                return True
            if len(responses) != len(running):
                for p in running:
                    p.future.set_exception(WorkerFailedError("collation returned the wrong number of responses"))
                return True
            for p, r in zip(running, responses):
                p.future.set_result(r)
            return True
        finally:
            lease.__exit__(None, None, None)
