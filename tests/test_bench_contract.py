"""The benchmark's reference arm on the CPU: one JSON line with the driver's
keys (metric, value, unit, steps, warmup, higher_is_better, impl, an e2e
object with zero host<->device bytes, a cpu_baseline describing the run), and
under torchrun a rank other than 0 exits 0 without output."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def _run(env_extra, *args):
    env = dict(os.environ, **env_extra)
    return subprocess.run([sys.executable, str(ROOT / "bench.py"), "--impl", "reference", *args],
                          capture_output=True, text=True, env=env, timeout=600, cwd=ROOT)


def test_reference_arm_prints_one_contract_line():
    r = _run({}, "--steps", "1", "--warmup", "0")
    assert r.returncode == 0, r.stderr[-2000:]
    lines = [x for x in r.stdout.splitlines() if x.startswith("{")]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d["impl"] == "reference" and d["metric"] == "scored requests/s" and d["unit"] == "requests/s"
    assert d["steps"] == 1 and d["warmup"] == 0 and d["higher_is_better"] is True and d["n_gpus"] == 1
    assert d["value"] > 0 and d["data"] == "synthetic" and "workload" in d["config"]
    assert d["e2e"] == {"value": d["value"], "unit": "requests/s", "h2d_bytes_per_step": 0,
                        "d2h_bytes_per_step": 0}
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] == "port" and cb["cores"] >= 1 and cb["sample"]


def test_reference_arm_other_ranks_exit_quietly():
    r = _run({"RANK": "1", "LOCAL_RANK": "1", "WORLD_SIZE": "2"}, "--steps", "1", "--warmup", "0", "--gpus", "2")
    assert r.returncode == 0, r.stderr[-2000:]
    assert not [x for x in r.stdout.splitlines() if x.startswith("{")]


def test_cpu_baseline_reports_rate_tokens_and_p50(synth_root):
    """The CPU leg of the GPU arm (oracle on a bounded sample) on a small model:
    requests/s, tokens/s and a p50 request latency over whole requests."""
    sys.path.insert(0, str(ROOT))
    import bench
    from huncho_b200 import synth
    d = synth.write_model(synth_root / "kev-mini-bf16", name="kev-mini", seed=0, store="bf16")
    wl = synth.make_workload(2, synth.SPECS["kev-mini"]["vocab_size"], seed=2, n_requests=3)
    order = [i for r in range(wl.n_requests) for i in range(len(wl.rows)) if wl.request_of[i] == r]
    cb = bench.cpu_baseline(d, "bf16", wl, order, max_seconds=60.0)
    assert cb["value"] > 0 and cb["tokens_per_s"] > 0 and cb["kind"] == "port" and cb["cores"] >= 1
    assert cb["p50_request_latency_ms"] > 0 and "3 requests" in cb["sample"]
    cp = bench.cpu_baseline(d, "bf16", wl, order, max_seconds=60.0, prefix_cache=True)
    assert cp["value"] > 0 and cp["p50_request_latency_ms"] > 0


def _bench():
    sys.path.insert(0, str(ROOT))
    import bench
    return bench


def test_pool_sharding_covers_every_request_once():
    """The multi-GPU bench splits ONE seeded pool by the batcher's token
    balance: every request on exactly one rank, its rows intact, per-rank
    tokens within one request of each other."""
    bench = _bench()
    from huncho_b200 import synth
    from huncho_b200.replicas import shard_by_tokens
    for world in (1, 2, 4, 8):
        pool = synth.make_workload(2, 248320, seed=0, n_requests=32 * world)
        toks = [0] * pool.n_requests
        for r, row in zip(pool.request_of, pool.rows):
            toks[r] += len(row)
        shards = shard_by_tokens(toks, world)
        parts = [bench.subset_workload(pool, sh) for sh in shards]
        assert sorted(i for sh in shards for i in sh) == list(range(pool.n_requests))
        assert sum(p.n_tokens for p in parts) == pool.n_tokens
        assert sum(len(p.rows) for p in parts) == len(pool.rows)
        loads = [p.n_tokens for p in parts]
        assert max(loads) - min(loads) <= max(toks)
        for p, sh in zip(parts, shards):
            assert set(p.request_of) == set(range(len(sh)))
            assert all(len(p.rows[i]) == toks[sh[p.request_of[i]]] // 3 for i in range(len(p.rows)))


def test_latency_summary_and_kernel_rooflines():
    bench = _bench()
    lat = bench.latency_summary([float(x) for x in range(1, 101)])
    assert lat["p50"] == 50.0 and lat["p95"] == 95.0 and lat["p99"] == 99.0 and lat["mean"] == 50.5
    pk = {"hbm_gbs": 6500.0, "bf16_tflops_sustained": 1300.0}
    prof = {"gemm": (10.0, 13e12, 1e9, 100), "rmsnorm": (1.0, 0.0, 6.5e9, 10), "attention": (0.0, 0.0, 0.0, 0)}
    rl = {e["class"]: e for e in bench.kernel_rooflines(prof, pk, "bf16")}
    assert set(rl) == {"gemm", "rmsnorm"}
    assert abs(rl["gemm"]["frac_tensor"] - 1.0) < 1e-9 and rl["gemm"]["bound"] == "tensor"
    assert abs(rl["rmsnorm"]["frac_hbm"] - 1.0) < 1e-9 and rl["rmsnorm"]["bound"] == "hbm"
    assert abs(rl["gemm"]["avg_ms"] - 0.1) < 1e-12
    # The kernels each class names follow the model dtype: the packed profiles'
    # projections are the tcgen05 kind::i8 GEMM, and their (fp32-activation)
    # attention and recurrence are the CUDA-core kernels.
    name, bound = bench.kernel_label("gemm", "q8_0-fp32")
    assert "gemm_q8_tc_kernel" in name and bound == "tensor"
    name, bound = bench.kernel_label("attention", "q4_0-fp32")
    assert "attn_simt_kernel" in name and bound != "tensor"
    assert "3xTF32" in bench.kernel_label("gemm", "fp32")[0]
    assert "attn_ws_kernel" in bench.kernel_label("attention", "bf16")[0]
    rl = {e["class"]: e for e in bench.kernel_rooflines(prof, pk, "q8_0-fp32")}
    assert "gemm_q8_tc_kernel" in rl["gemm"]["kernel"]


def test_cpu_legs_use_every_core_under_torchrun_threads():
    """torchrun exports OMP_NUM_THREADS=1; the CPU legs still run BLAS on all
    host cores and say so."""
    code = ("import sys; sys.path.insert(0, %r); import bench; from threadpoolctl import threadpool_info; "
            "c = bench.host_cores()\n"
            "with bench.use_all_cores(c):\n"
            "    n = [i['num_threads'] for i in threadpool_info() if i['user_api'] == 'blas']\n"
            "print(c, min(n))" % str(ROOT))
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True, timeout=300, cwd=ROOT,
                       env=dict(os.environ, OMP_NUM_THREADS="1"))
    assert r.returncode == 0, r.stderr[-2000:]
    cores, blas = map(int, r.stdout.split())
    assert blas == cores
