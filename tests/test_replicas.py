"""Host side of the multi-GPU path on CPU: the request shard plan, the replica
pool (crates/huncho-api/src/replicas.rs:7-61), and world-size-2 `gloo` ranks
scoring their shares and meeting on rank 0 (the torchrun layout of the bench,
with a host scorer standing in for the GPU backend)."""
import os
import socket
import threading

import numpy as np
import pytest

from huncho_b200.replicas import ReplicaPool, gather_to_rank0, max_over_ranks, score_sharded, shard_by_tokens


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_shard_plan_covers_every_request_once_and_balances_tokens(world):
    rng = np.random.default_rng(world)
    lengths = rng.integers(32, 2048, 257).tolist()
    plan = shard_by_tokens(lengths, world)
    assert len(plan) == world
    flat = sorted(i for s in plan for i in s)
    assert flat == list(range(len(lengths)))
    assert all(s == sorted(s) for s in plan)
    loads = [sum(lengths[i] for i in s) for s in plan]
    # Greedy longest-first: no rank exceeds another by more than one request.
    assert max(loads) - min(loads) <= max(lengths)
    assert plan == shard_by_tokens(list(lengths), world)  # every rank computes the same plan


def test_shard_plan_edge_cases():
    assert shard_by_tokens([], 4) == [[], [], [], []]
    assert shard_by_tokens([5], 3) == [[0], [], []]
    assert shard_by_tokens([7, 7, 7, 7], 2) == [[0, 2], [1, 3]]
    with pytest.raises(ValueError):
        shard_by_tokens([1], 0)
    with pytest.raises(ValueError):
        shard_by_tokens([-1], 1)


def test_replica_pool_leases_lowest_idle_first_and_returns_on_error():
    pool = ReplicaPool(["a", "b", "c"])
    with pool.lease() as x:
        assert x == "a"
        with pool.lease() as y:
            assert y == "b"
    with pytest.raises(KeyError):
        with pool.lease() as x:
            assert x == "a"
            raise KeyError("job failed")
    with pool.lease() as x:  # returned despite the exception
        assert x == "a"
    with pytest.raises(ValueError):
        ReplicaPool([])


def test_replica_pool_blocks_until_idle_and_closes():
    pool = ReplicaPool(["only"])
    seen, order = [], []
    gate = threading.Event()

    def worker(k):
        with pool.lease() as b:
            order.append(("in", k))
            seen.append(b)
            gate.wait(1.0)
            order.append(("out", k))

    ts = [threading.Thread(target=worker, args=(k,)) for k in range(3)]
    for t in ts:
        t.start()
    gate.set()
    for t in ts:
        t.join(5.0)
    assert seen == ["only"] * 3
    # One lease at a time: every "in" is followed by its own "out".
    assert all(order[i][0] == "in" and order[i + 1] == ("out", order[i][1]) for i in range(0, 6, 2))
    with pool.lease():
        with pytest.raises(TimeoutError):
            with pool.lease(timeout=0.05):
                pass
    pool.close()
    with pytest.raises(RuntimeError):
        with pool.lease(timeout=0.05):
            pass


def test_single_process_gather_and_max():
    assert gather_to_rank0(["x", "y"], [1, 0], 2) == ["y", "x"]
    assert max_over_ranks(2.5) == 2.5
    assert score_sharded(lambda idx: [i * 10 for i in idx], [3, 1, 2]) == [0, 10, 20]


def _fake_score(rows):
    """A deterministic stand-in for a backend's per-request result."""
    return [float(sum(r)) / len(r) for r in rows]


def _rank_main(rank, world, port, out_dir, fail_rank):
    import torch.distributed as dist
    from datetime import timedelta
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        rng = np.random.default_rng(11)
        rows = [rng.integers(0, 1000, int(n)).tolist() for n in rng.integers(1, 300, 37)]
        lengths = [len(r) for r in rows]
        mine = []

        def score(idx):
            mine.extend(idx)
            if rank == fail_rank:
                raise RuntimeError("rank failed")
            return _fake_score([rows[i] for i in idx])

        try:
            got = score_sharded(score, lengths)
        except RuntimeError as e:
            if rank == fail_rank:  # leave between steps, nothing in flight
                os._exit(3)
            raise e
        slowest = max_over_ranks(1.0 + rank)
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(repr({"mine": mine, "got": got, "expect": _fake_score(rows) if rank == 0 else None,
                          "slowest": slowest, "plan": shard_by_tokens(lengths, world)[rank]}))
    except Exception as e:  # the surviving rank records how it learned of the failure
        with open(os.path.join(out_dir, f"rank{rank}.txt"), "w") as f:
            f.write(repr({"error": type(e).__name__}))
    finally:
        if dist.is_initialized():
            try:
                dist.destroy_process_group()
            except Exception:
                pass


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _spawn(tmp_path, fail_rank):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, str(tmp_path), fail_rank)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(120)
        if p.is_alive():
            p.kill()
            pytest.fail("a gloo rank did not finish")
    return procs


def test_gloo_two_ranks_score_their_shares_and_meet_on_rank0(tmp_path):
    procs = _spawn(tmp_path, fail_rank=-1)
    assert [p.exitcode for p in procs] == [0, 0]
    r0 = eval((tmp_path / "rank0.txt").read_text())
    r1 = eval((tmp_path / "rank1.txt").read_text())
    assert r0["got"] == r0["expect"]
    assert r1["got"] is None
    assert sorted(r0["mine"] + r1["mine"]) == list(range(37))
    assert r0["mine"] == r0["plan"] and r1["mine"] == r1["plan"]
    assert r0["slowest"] == r1["slowest"] == 2.0


def test_gloo_rank_failure_reaches_the_other_rank_on_the_host(tmp_path):
    procs = _spawn(tmp_path, fail_rank=1)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 0
    assert "error" in eval((tmp_path / "rank0.txt").read_text())
