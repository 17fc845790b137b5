"""Replicas: the scoring path spread over GPUs with no data-path collective.

Requests are independent (`forward_independent_batch`,
crates/huncho-backend/src/qwen3_5.rs:3138-3194; no cross-row attention,
crates/huncho-backend/src/backend.rs:245-246), so the path shards by request:

* inside one process, `ReplicaPool` leases idle backends (one per GPU, or
  several per GPU from `KevBackend.replica`) to callers for a whole job, as the
  reference's pool does (crates/huncho-api/src/replicas.rs:7-61);
* across processes (one per GPU under torchrun), every rank computes the same
  `shard_by_tokens` plan from the request lengths alone, scores its own share,
  and the host results meet on rank 0 (`gather_to_rank0`). The only
  collectives are host-side: the plan needs none, results travel as Python
  objects, and timing takes the max over ranks.
"""
from __future__ import annotations

import heapq
import threading
from contextlib import contextmanager
from typing import Callable, List, Optional, Sequence

__all__ = ["shard_by_tokens", "ReplicaPool", "gather_to_rank0", "max_over_ranks", "score_sharded"]


def shard_by_tokens(lengths: Sequence[int], world: int) -> List[List[int]]:
    """Per-rank request indices, greedily balanced by total tokens.

    Longest request first, each to the rank with the fewest tokens so far
    (ties: the lower rank); each rank's list is returned in request order.
    The plan depends only on `lengths` and `world`, so every rank computes it
    alone and all ranks agree.
    """
    if world < 1:
        raise ValueError("world must be >= 1")
    if any(int(n) < 0 for n in lengths):
        raise ValueError("request lengths must be non-negative")
    heap = [(0, r) for r in range(world)]
    shards: List[List[int]] = [[] for _ in range(world)]
    for i in sorted(range(len(lengths)), key=lambda i: (-int(lengths[i]), i)):
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + int(lengths[i]), r))
    return [sorted(s) for s in shards]


class ReplicaPool:
    """Idle backends leased for a whole job (replicas.rs:7-61).

    `lease()` blocks until a backend is idle and hands out the lowest idle
    index first (the reference's idle stack starts reversed, replicas.rs:16);
    the backend returns to the pool when the `with` block ends, exception or
    not. A closed pool refuses new leases.
    """

    def __init__(self, backends: Sequence):
        if not backends:
            raise ValueError("a replica pool needs at least one backend")
        self.backends = list(backends)
        self._idle = list(range(len(self.backends)))[::-1]
        self._cv = threading.Condition()
        self._closed = False

    def __len__(self) -> int:
        return len(self.backends)

    def close(self) -> None:
        with self._cv:
            self._closed = True
            self._cv.notify_all()

    @contextmanager
    def lease(self, timeout: Optional[float] = None):
        with self._cv:
            if not self._cv.wait_for(lambda: self._closed or self._idle, timeout=timeout):
                raise TimeoutError("no idle replica")
            if self._closed:
                raise RuntimeError("replica pool is closed")
            index = self._idle.pop()
        try:
            yield self.backends[index]
        finally:
            with self._cv:
                self._idle.append(index)
                self._idle.sort(reverse=True)
                self._cv.notify()


def _dist():
    import torch.distributed as dist
    return dist


def gather_to_rank0(local: list, shard: Sequence[int], n_total: int, group=None) -> Optional[list]:
    """Every rank's per-request results back in request order on rank 0 (None
    elsewhere). `local[k]` is the result of request `shard[k]`."""
    dist = _dist()
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        out = [None] * n_total
        for i, v in zip(shard, local):
            out[i] = v
        return out
    rank = dist.get_rank(group)
    parts = [None] * dist.get_world_size(group) if rank == 0 else None
    dist.gather_object((list(shard), list(local)), parts, dst=0, group=group)
    if rank != 0:
        return None
    out = [None] * n_total
    for idx, vals in parts:
        for i, v in zip(idx, vals):
            out[i] = v
    if any(v is None for v in out):
        raise RuntimeError("a request was scored by no rank")
    return out


def max_over_ranks(value: float, group=None) -> float:
    """The maximum of a host float over the ranks (device timing of a step is
    the slowest rank's). The reduction runs on the CPU under gloo and on the
    rank's GPU under NCCL."""
    dist = _dist()
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return float(value)
    import torch
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())


def score_sharded(score: Callable[[List[int]], list], lengths: Sequence[int], group=None) -> Optional[list]:
    """Score requests spread over the ranks: `score(indices)` scores this
    rank's share (a list with one result per index); rank 0 gets all results
    in request order."""
    dist = _dist()
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    rank = dist.get_rank(group) if dist.is_initialized() else 0
    shard = shard_by_tokens(lengths, world)[rank]
    local = score(shard) if shard else []
    if len(local) != len(shard):
        raise RuntimeError("score() must return one result per request")
    return gather_to_rank0(local, shard, len(lengths), group)
