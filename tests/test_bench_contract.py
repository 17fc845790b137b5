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
