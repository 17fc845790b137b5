#!/usr/bin/env python
"""Kev scoring throughput on B200: scored requests/s, prompt tokens/s, p50 latency.

Workload (default, config 2 of the benchmark definition): the Qwen3.5-0.8B-shaped
Kev scorer in bf16 (random-init weights from a fixed seed), 32 requests with
lengths uniform in [64, 512]; each asks a 4-option choice, a noul and a 5-level
score, so one step scores 96 independent rows (~27.6k prompt tokens) split into
two native batches of 48 rows. Each GPU holds `--replicas` (default 2) model
handles (hk_replica on the same GPU: one shared copy of the weights, each
handle with its own workspace and CUDA stream); a step's native batches are dealt to them round-robin and run
concurrently, so one batch's kernel tails and launch gaps overlap the other's
work. Under torchrun one request pool is generated from one seed (32 requests
per GPU for configs 1-4: weak scaling; config 5's fixed 4096 requests: strong
scaling) and split over the ranks by `replicas.shard_by_tokens`, the batcher's
token-balanced plan; each rank (one per GPU) scores its share (replicas, no
collective on the data path).

  value  device time of K steps with inputs resident in HBM (hk_score_device),
         L2 flushed between steps (256 MiB write, outside the timed events);
  e2e    the same K steps through the public host API (KevBackend.score_answers
         -> hk_score_answers: host->device copy of the inputs, forward,
         calibration and answer fields on the device, device->host read of the
         probabilities and answers; one host thread per replica), plus the
         answer dicts, wall clock;
both are the max over ranks. The kernel roofline comes from a serial pass of
the same K steps (one handle, one stream) with per-launch CUDA events, since
launches on concurrent streams overlap. `--impl reference` times the CPU reference path
(the oracle restatement of the reference's CPU fp32 forward) on rank 0.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

from huncho_b200 import calibration, engine, synth  # noqa: E402
from huncho_b200.backend import pack_rows  # noqa: E402

CLOCK_QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
               "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
               "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class ClockSampler:
    """nvidia-smi samples of one GPU while the timed region runs."""

    def __init__(self, index: int):
        self.index = index
        self.proc = None

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={CLOCK_QUERY}", "--format=csv,noheader",
                                          "-i", str(self.index), "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        self.lines = []
        if self.proc:
            time.sleep(0.25)
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                out, _ = self.proc.communicate()
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1].split()[0]))
                mx = float(f[2].split()[0])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


WORKLOADS = {
    1: "cfg1: Kev-0.8B {dtype}, {n} request x 256 tokens, one 4-option choice",
    2: "cfg2: Kev-0.8B {dtype}, {n} requests per GPU x 3 questions (choice-4, noul, score-5), lengths U[64,512], "
       "packed varlen",
    3: "cfg3: Kev-0.8B int8 per-channel weights, {n} requests per GPU x 1024 tokens, 8-option choice",
    4: "cfg4: Kev-0.8B {dtype}, {n} requests per GPU x 8192 tokens, noul; KV in 16-token pages, shuffled block table",
    5: "cfg5: Kev-4B {dtype}, {n} requests per GPU, lengths log-uniform [32, 2048], mixed questions",
}


def groups_of(rows, limit=64):
    """Split rows into the fewest native batches of at most `limit` rows, equal-sized."""
    n = len(rows)
    k = -(-n // limit)
    size = -(-n // k)
    return [list(range(i, min(n, i + size))) for i in range(0, n, size)]


def request_plan(wl):
    """Per request: its shared prefix (the longest common prefix of its rows
    that leaves every readout in the suffix) and, per question row, the suffix
    and suffix-relative positions (the engine's prefix_cache fan-out,
    eng:878-960)."""
    by_req = {}
    for i, r in enumerate(wl.request_of):
        by_req.setdefault(r, []).append(i)
    plan = []
    for key in sorted(by_req):
        q = by_req[key]
        rows_q = [wl.rows[i] for i in q]
        p = min(len(r) for r in rows_q)
        for r in rows_q[1:]:
            p = min(p, next((j for j, (x, y) in enumerate(zip(rows_q[0], r)) if x != y), p))
        p = min([p] + [min(wl.positions[i]) for i in q])
        plan.append((list(rows_q[0][:p]), [(i, list(wl.rows[i][p:]), [x - p for x in wl.positions[i]]) for i in q]))
    return plan


# Kernel (class) names of the half-precision models' forward, by profile class.
KERNEL_NAMES = {
    "gemm": "gemm_f16_tc_kernel + gemm_f16_tc2_kernel (tcgen05 projections)",
    "delta": "delta_pipe_kernel (fused delta layer: conv, gates, chunked rule, gated norm)",
    "attention": "attn_ws_kernel (warp-specialised tcgen05 causal GQA attention; attn_t5_kernel for prefix rows)",
    "delta_prep": "delta_prep_vec_kernel (fp32 model's delta input stage)",
    "other": "swiglu / gated_norm / conv_history kernels",
    "rmsnorm": "rmsnorm_reg_kernel",
    "attn_prep": "attn_prep_vec_kernel (q/k norm, partial RoPE, K/V store)",
    "readout": "readout_norm / readout_proj / pointer_logits kernels",
    "embed": "embed_kernel",
}
TENSOR_CLASSES = ("gemm", "delta", "attention")
# The fp32-activation paths (the fp32 model and the packed profiles) run other
# kernels in some classes.
FP32_ACT_KERNELS = {
    "delta": "delta_recurrent_kernel (the reference's per-token order, fp32)",
    "attention": "attn_simt_kernel (fp32 causal GQA attention on CUDA cores)",
}
PACKED_DTYPES = ("q8_0-fp32", "q4_0-fp32")


def kernel_label(cls, dtype):
    """(kernel name, bound) of a profile class under a model dtype."""
    if cls == "gemm" and dtype in PACKED_DTYPES:
        return ("quantize_rows_kernel + gemm_q8_tc_kernel (tcgen05 kind::i8 packed projections, block scales "
                "in the epilogue; int8 ops against the bf16 peak, no measured int8 peak)", "tensor")
    if cls == "gemm" and dtype == "fp32":
        return "gemm_f16_tc_kernel (3xTF32 projections: three kind::tf32 products per tile)", "tensor"
    if (dtype == "fp32" or dtype in PACKED_DTYPES) and cls in FP32_ACT_KERNELS:
        return FP32_ACT_KERNELS[cls], "fp32 CUDA cores"
    return KERNEL_NAMES.get(cls, cls), "tensor" if cls in TENSOR_CLASSES else "hbm"


def kernel_rooflines(prof, pk, dtype):
    """One entry per kernel class that launched: launches, average CUDA-event
    time per launch, algorithmic FLOPs and HBM bytes per launch, achieved
    TFLOP/s and GB/s, and the fractions of the measured peaks (sustained bf16
    tensor peak; HBM copy bandwidth). `bound` names the roofline that limits
    the kernel's design."""
    out = []
    total_ms = sum(v[0] for v in prof.values()) or 1.0
    for cls, (ms, fl, by, n) in prof.items():
        if not n or ms <= 0:
            continue
        sec = ms / 1e3
        name, bound = kernel_label(cls, dtype)
        e = {"kernel": name, "class": cls, "launches": int(n), "avg_ms": ms / n,
             "share": round(ms / total_ms, 4), "bound": bound}
        if fl:
            e["flops_per_launch"] = fl / n
            e["achieved_tflops"] = fl / sec / 1e12
            e["frac_tensor"] = e["achieved_tflops"] / pk["bf16_tflops_sustained"]
        if by:
            e["bytes_per_launch"] = by / n
            e["achieved_gbs"] = by / sec / 1e9
            e["frac_hbm"] = e["achieved_gbs"] / pk["hbm_gbs"]
        out.append(e)
    return out


def latency_summary(step_ms):
    """Mean and nearest-rank p50 / p95 / p99 of the step times (every request
    of a step completes when its step ends); the shape of the reference's
    bench report (crates/huncho-cli/src/bench.rs:290-315)."""
    xs = sorted(step_ms)

    def pct(p):
        return xs[min(len(xs) - 1, max(0, int(np.ceil(p / 100.0 * len(xs))) - 1))]

    return {"mean": statistics.mean(xs), "p50": pct(50), "p95": pct(95), "p99": pct(99), "n": len(xs)}


def subset_workload(pool, requests):
    """The rows of `requests` (indices into the pool), renumbered 0.."""
    keep = {r: k for k, r in enumerate(requests)}
    idx = [i for i, r in enumerate(pool.request_of) if r in keep]
    return synth.Workload(name=pool.name, rows=[pool.rows[i] for i in idx],
                          positions=[pool.positions[i] for i in idx], qtypes=[pool.qtypes[i] for i in idx],
                          request_of=[keep[pool.request_of[i]] for i in idx], n_requests=len(requests))


def model_dir_for(name, store, seed):
    return synth.default_dir(name, seed, store)


def host_cores() -> int:
    """Host cores this process may run on."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def use_all_cores(cores: int):
    """Let the CPU legs use every host core: the oracle's C recurrence threads
    and NumPy's BLAS pool (torchrun exports OMP_NUM_THREADS=1, which would
    otherwise leave BLAS on one thread). Returns the BLAS limiter (a context
    manager)."""
    from oracle import kev_oracle as ko
    from threadpoolctl import threadpool_limits
    ko.set_threads(cores)
    return threadpool_limits(limits=cores, user_api="blas")


def cpu_baseline(model_dir, dtype, wl, rows_idx, max_seconds=30.0, prefix_cache=False):
    """The CPU oracle on a bounded sample of the workload (whole rows; with
    prefix_cache whole requests: prefix once, each question as a branch)."""
    cores = host_cores()
    with use_all_cores(cores):
        return _cpu_baseline(model_dir, dtype, wl, rows_idx, max_seconds, prefix_cache, cores)


def _cpu_baseline(model_dir, dtype, wl, rows_idx, max_seconds, prefix_cache, cores):
    from oracle import kev_oracle as ko
    m = ko.load_model(model_dir, dtype)
    if prefix_cache:
        t0 = time.perf_counter()
        done, toks, lat = 0, 0, []
        for prefix, qs in request_plan(wl):
            ts = time.perf_counter()
            cache = ko.prefill(m, prefix)
            for i, suf, sp in qs:
                ko.calibrate(ko.score_branch(m, cache, suf, sp), m.temperature)
                toks += len(wl.rows[i])
            lat.append(time.perf_counter() - ts)
            done += 1
            if time.perf_counter() - t0 > max_seconds:
                break
        dt = time.perf_counter() - t0
        return {"value": done / dt, "unit": "requests/s", "cores": cores, "kind": "port",
                "tokens_per_s": toks / dt, "p50_request_latency_ms": 1000.0 * statistics.median(lat),
                "sample": f"{done} whole requests ({toks} prompt tokens) of the workload, CPU fp32 oracle with "
                          f"prefix caches (prefix once, each question a branch) on the same weights, {dt:.1f} s"}
    t0 = time.perf_counter()
    done, toks = 0, 0
    need = {}  # rows per request, and each request's CPU time once all its rows ran
    for r in wl.request_of:
        need[r] = need.get(r, 0) + 1
    spent, seen, lat = {}, {}, []
    for i in rows_idx:
        ts = time.perf_counter()
        ko.calibrate(ko.score_row(m, wl.rows[i], wl.positions[i]), m.temperature)
        r = wl.request_of[i]
        spent[r] = spent.get(r, 0.0) + time.perf_counter() - ts
        seen[r] = seen.get(r, 0) + 1
        if seen[r] == need[r]:
            lat.append(spent[r])
        done += 1
        toks += len(wl.rows[i])
        if time.perf_counter() - t0 > max_seconds:
            break
    dt = time.perf_counter() - t0
    rows_per_req = len(wl.rows) / wl.n_requests
    return {"value": (done / rows_per_req) / dt, "unit": "requests/s", "cores": cores, "kind": "port",
            "tokens_per_s": toks / dt,
            "p50_request_latency_ms": 1000.0 * statistics.median(lat) if lat else None,
            "sample": f"{done} question rows ({toks} tokens) of the workload, CPU fp32 oracle on the same weights, "
                      f"{dt:.1f} s; p50 latency over the {len(lat)} requests whose rows all ran"}


def reference_arm(args, rank, world):
    if rank != 0:
        return 0
    cores = host_cores()
    with use_all_cores(cores):
        return _reference_arm(args, cores)


def _reference_arm(args, cores):
    from oracle import kev_oracle as ko
    name, store, dtype = "kev-0.8b", "bf16", "bf16"
    d = synth.write_model(model_dir_for(name, store, args.seed), name, args.seed, store)
    m = ko.load_model(d, dtype)
    wl = synth.make_workload(args.config, m.cfg.vocab_size, seed=args.seed)
    rows_per_req = len(wl.rows) / wl.n_requests
    times, toks = [], 0
    if args.prefix_cache:
        plan = request_plan(wl)
        for s in range(args.warmup + args.steps):
            prefix, qs = plan[s % len(plan)]
            t0 = time.perf_counter()
            cache = ko.prefill(m, prefix)
            for i, suf, sp in qs:
                ko.calibrate(ko.score_branch(m, cache, suf, sp), m.temperature)
            if s >= args.warmup:
                times.append(time.perf_counter() - t0)
                toks += sum(len(wl.rows[i]) for i, _, _ in qs)
        total = sum(times)
        value = len(times) / total
        line = {
            "impl": "reference", "metric": "scored requests/s", "value": value, "unit": "requests/s",
            "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "prompt_tokens_per_s": toks / total,
            "config": {"workload": f"cfg{args.config}: Kev-0.8B, 32 requests x (choice-4, noul, score-5), lengths "
                                   "U[64,512]; prefix cache: each request's shared prefix once, questions as branches",
                       "model": "kev-0.8b (bf16 weights, fp32 math)", "step": "one whole request per step"},
            "cpu_baseline": {"value": value, "unit": "requests/s", "cores": cores, "kind": "port",
                             "sample": f"{len(times)} whole requests, {toks} prompt tokens; the CPU oracle restating "
                                       "the reference CPU fp32 Kev forward with its prefix caches (the Rust reference "
                                       "cannot be built here)"},
            "e2e": {"value": value, "unit": "requests/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        print(json.dumps(line))
        return 0
    for s in range(args.warmup + args.steps):
        i = s % len(wl.rows)
        t0 = time.perf_counter()
        ko.calibrate(ko.score_row(m, wl.rows[i], wl.positions[i]), m.temperature)
        if s >= args.warmup:
            times.append(time.perf_counter() - t0)
            toks += len(wl.rows[i])
    total = sum(times)
    value = (len(times) / rows_per_req) / total
    line = {
        "impl": "reference", "metric": "scored requests/s", "value": value, "unit": "requests/s",
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * total / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "prompt_tokens_per_s": toks / total,
        "config": {"workload": f"cfg{args.config}: Kev-0.8B, 32 requests x (choice-4, noul, score-5), "
                                "lengths U[64,512]", "model": "kev-0.8b (bf16 weights, fp32 math)",
                   "step": "one question row (1/3 request) per step"},
        "cpu_baseline": {"value": value, "unit": "requests/s", "cores": cores, "kind": "port",
                         "sample": f"{len(times)} question rows, {toks} tokens; the CPU oracle restating the "
                                   "reference CPU fp32 Kev forward (the Rust reference cannot be built here)"},
        "e2e": {"value": value, "unit": "requests/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line))
    return 0


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=10)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--config", type=int, default=2)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--requests", type=int, default=None,
                    help="requests per GPU (default: the config's); smaller cases are for profiling")
    ap.add_argument("--packed", choices=["q8_0-fp32", "q4_0-fp32"], default=None,
                    help="run the workload on the reference's packed profile: the synthetic model converted "
                         "(fp32 weights, projections in GGML Q8_0 / Q4_0 blocks, fp32 activations)")
    ap.add_argument("--replicas", type=int, default=2,
                    help="model handles per GPU (shared weights; each its own workspace and stream); the step's native "
                         "batches run on them concurrently (1 = one handle, batches in sequence)")
    ap.add_argument("--prefix-cache", action="store_true",
                    help="score each request's questions as branches of its cached shared prefix (the reference "
                         "engine's prefix_cache option: prefill + fork); default: independent rows")
    args = ap.parse_args()
    rank = int(os.environ.get("RANK", 0))
    world = int(os.environ.get("WORLD_SIZE", 1))
    local = int(os.environ.get("LOCAL_RANK", 0))
    if args.impl == "reference":
        return reference_arm(args, rank, world)

    import torch
    import torch.distributed as dist
    from datetime import timedelta
    from huncho_b200.backend import KevBackend

    torch.cuda.set_device(local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    from huncho_b200.replicas import max_over_ranks

    name, store = ("kev-0.8b", "bf16")
    dtype = {1: "fp32", 2: "bf16", 3: "int8w", 4: "bf16"}.get(args.config, "bf16")
    if args.config == 1 or args.packed:
        store = "fp32"
    if args.config == 5:
        name = "kev-4b"
    d = model_dir_for(name, store, args.seed)
    if rank == 0:
        synth.write_model(d, name, args.seed, store)
    if args.packed:
        from huncho_b200 import quantize
        dtype = args.packed
        pd = Path(str(d) + "-" + args.packed)
        if rank == 0 and not (pd / "backbone.gguf").exists():
            quantize.write_package(d, args.packed, pd)
        d = pd
    barrier()
    from huncho_b200.replicas import shard_by_tokens
    # One request pool from one seed, split over the ranks by the batcher's
    # token-balanced plan: 32 (cfg 2) requests per GPU for configs 1-4 (weak
    # scaling), config 5's fixed pool of 4096 requests (strong scaling).
    strong = args.config == 5
    per_gpu = args.requests or {1: 1, 2: 32, 3: 64, 4: 8, 5: 4096}[args.config]
    req_pool = synth.make_workload(args.config, synth.SPECS[name]["vocab_size"], seed=args.seed,
                                   n_requests=per_gpu if strong else per_gpu * world)
    req_tokens = [0] * req_pool.n_requests
    for r, row in zip(req_pool.request_of, req_pool.rows):
        req_tokens[r] += len(row)
    wl = subset_workload(req_pool, shard_by_tokens(req_tokens, world)[rank])
    max_len = max(len(r) for r in wl.rows)
    backend = KevBackend(d, device=local, dtype=dtype, max_context=max(8192, max_len))
    if args.config == 4:
        backend.with_kv_page_tokens(16, shuffle_seed=1 + rank)  # 16-token pages, shuffled block table

    groups = groups_of(wl.rows, backend.batch_limits().max_rows)
    n_rep = max(1, min(args.replicas, len(wl.rows)))
    if args.prefix_cache:
        n_rep = 1  # the prefix-cache step is synchronous host code on one handle
    if n_rep > len(groups):  # at least one native batch per replica
        size = -(-len(wl.rows) // n_rep)
        groups = [list(range(i, min(len(wl.rows), i + size))) for i in range(0, len(wl.rows), size)]
    n_rep = min(n_rep, len(groups))
    backends = [backend] + [backend.replica() for _ in range(n_rep - 1)]
    if args.config == 4:
        for k, b in enumerate(backends[1:]):
            b.with_kv_page_tokens(16, shuffle_seed=2 + k + rank)
    packed = []
    for g in groups:
        tok, cu, pos, cup = pack_rows([wl.rows[i] for i in g], [wl.positions[i] for i in g])
        dev = {"tok": torch.from_numpy(tok.view(np.int32)).cuda(), "cu": torch.from_numpy(cu).cuda(),
               "pos": torch.from_numpy(pos).cuda(), "out": torch.empty(int(cup[-1]), device="cuda")}
        packed.append((g, tok, cu, pos, cup, dev))
    n_tok = wl.n_tokens
    flush = torch.empty(256 * 1024 * 1024 // 4, dtype=torch.float32, device="cuda")
    # A dedicated stream: the forward, the L2 flush and the timing events all
    # run on it (the legacy default stream has no handle to pass).
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)

    rep_streams = [torch.cuda.Stream() for _ in range(n_rep)]

    def serial_step():
        for g, tok, cu, pos, cup, dev in packed:
            backend.score_device(cu, cup, dev["tok"].data_ptr(), dev["cu"].data_ptr(), dev["pos"].data_ptr(),
                                 dev["out"].data_ptr(), stream.cuda_stream)

    def device_step():
        if n_rep == 1:
            serial_step()
            return
        # Fork the replica streams off the timing stream and join them back.
        go = torch.cuda.Event()
        go.record(stream)
        for rs in rep_streams:
            rs.wait_event(go)
        for j, (g, tok, cu, pos, cup, dev) in enumerate(packed):
            backends[j % n_rep].score_device(cu, cup, dev["tok"].data_ptr(), dev["cu"].data_ptr(),
                                             dev["pos"].data_ptr(), dev["out"].data_ptr(),
                                             rep_streams[j % n_rep].cuda_stream)
        for rs in rep_streams:
            done = torch.cuda.Event()
            done.record(rs)
            stream.wait_event(done)

    # Prefix-cache mode: per request, the longest common prefix of its rows
    # that leaves every readout in the suffix is prefilled once; each question
    # is then scored as a branch of it (eng:878-960 with prefix_cache).
    fork_plan = None
    if args.prefix_cache:
        from huncho_b200 import _native
        prefixes, suffixes = [], []
        for prefix, qs in request_plan(wl):
            prefixes.append(prefix)
            for i, suf, sp in qs:
                suffixes.append((len(prefixes) - 1, i, suf, sp))
        lim = _native.HK_MAX_CACHED_ROWS
        pre_groups = [list(range(a, min(len(prefixes), a + lim))) for a in range(0, len(prefixes), lim)]
        row_groups = [suffixes[a:a + lim] for a in range(0, len(suffixes), lim)]
        packed_rows = [(grp, pack_rows([x[2] for x in grp], [x[3] for x in grp])) for grp in row_groups]
        fork_plan = (prefixes, pre_groups, packed_rows)

    def fork_step(answers: bool):
        prefixes, pre_groups, packed_rows = fork_plan
        handles = []
        for g in pre_groups:
            handles += backend.prefill_batch([prefixes[j] for j in g])
        for grp, args_ in packed_rows:
            logits, _ = backend.score_cached(*args_, parents=[handles[x[0]] for x in grp],
                                             mode=_native.HK_CACHE_BRANCH)
            if answers:
                cup = args_[3]
                for j, x in enumerate(grp):
                    lo, hi = int(cup[j]), int(cup[j + 1])
                    probs = calibration.calibrate(logits[lo:hi], backend.temperature)
                    q = engine.Question(wl.qtypes[x[1]], labels=[str(v) for v in range(hi - lo)],
                                        descriptions=["" for _ in range(hi - lo)])
                    engine.build_answer(q, engine.candidates_for(q, wl.positions[x[1]]), probs)
        for h in handles:
            backend.release_cache(h)

    if fork_plan is not None:
        def device_step():  # noqa: F811 -- the native calls synchronise; timed on the host clock
            fork_step(False)

    # warm-up (also sizes the workspace)
    for _ in range(args.warmup):
        flush.zero_()
        device_step()
    torch.cuda.synchronize()

    # ---- timed region: device-resident inputs
    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    launches0 = sum(b.kernel_launches for b in backends)
    backend.profile(fork_plan is None and n_rep == 1)
    barrier()
    torch.cuda.synchronize()
    host_ms = []
    with ClockSampler(local) as clk:
        for k in range(args.steps):
            flush.zero_()
            if fork_plan is not None:
                torch.cuda.synchronize()
                ts = time.perf_counter()
                device_step()
                host_ms.append(1000.0 * (time.perf_counter() - ts))
                continue
            starts[k].record(stream)
            device_step()
            ends[k].record(stream)
        torch.cuda.synchronize()
    barrier()
    backend.profile(False)
    prof = backend.profile_read()
    launches = sum(b.kernel_launches for b in backends) - launches0
    step_ms = host_ms if fork_plan is not None else [s.elapsed_time(e) for s, e in zip(starts, ends)]
    dev_total_s = max_over_ranks(sum(step_ms) / 1000.0)

    # ---- serial pass for the kernel roofline: the same steps on one handle and
    # one stream, each launch bracketed by CUDA events (concurrent streams would
    # make those intervals overlap).
    serial_ms = None
    if n_rep > 1:
        s_starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        s_ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
        serial_step()  # sizes the first handle's workspace for every batch
        torch.cuda.synchronize()
        backend.profile(True)
        for k in range(args.steps):
            flush.zero_()
            s_starts[k].record(stream)
            serial_step()
            s_ends[k].record(stream)
        torch.cuda.synchronize()
        backend.profile(False)
        prof = backend.profile_read()
        serial_ms = [a.elapsed_time(b) for a, b in zip(s_starts, s_ends)]

    # ---- e2e: the public host API, host calibration and answers included
    # e2e per native batch: inputs + question types up; probabilities, answer
    # records (16 bytes per row) and the error word down.
    h2d = sum(tok.nbytes + cu.nbytes + pos.nbytes + cup.nbytes + 4 * len(g) for g, tok, cu, pos, cup, _ in packed)
    d2h = sum(4 * int(cup[-1]) + 16 * len(g) + 4 for g, _, _, _, cup, _ in packed)

    if fork_plan is not None:
        h2d = sum(4 * len(p) + 8 for p in fork_plan[0]) + sum(
            a[0].nbytes + a[1].nbytes + a[2].nbytes + a[3].nbytes + 8 * len(g) for g, a in fork_plan[2])
        d2h = sum(4 * int(a[3][-1]) + 4 for _, a in fork_plan[2]) + 8 * len(fork_plan[0])

    def e2e_batches(r):
        # Replica r's native batches, one call each: forward + on-device
        # calibration and answers (the call releases the GIL while it runs).
        out = []
        for j in range(r, len(packed), n_rep):
            g, tok, cu, pos, cup, _ = packed[j]
            probs, rec = backends[r].score_answers(tok, cu, pos, cup, [wl.qtypes[i] for i in g])
            out.append((g, cup, probs, rec))
        return out

    pool = ThreadPoolExecutor(max_workers=n_rep) if n_rep > 1 else None

    def e2e_step():
        if fork_plan is not None:
            fork_step(True)
            return
        done = (list(pool.map(e2e_batches, range(n_rep))) if pool is not None else [e2e_batches(0)])
        for g, cup, probs, rec in (x for part in done for x in part):
            for j, i in enumerate(g):
                lo, hi = int(cup[j]), int(cup[j + 1])
                q = engine.Question(wl.qtypes[i], labels=[str(x) for x in range(hi - lo)],
                                    descriptions=["" for _ in range(hi - lo)])
                engine.answer_from_record(q, engine.candidates_for(q, wl.positions[i]), probs[lo:hi], rec[j])

    e2e_step()
    barrier()
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    e2e_times = []
    for _ in range(args.steps):
        ts = time.perf_counter()
        e2e_step()
        e2e_times.append(time.perf_counter() - ts)
    e2e_total_s = max_over_ranks(time.perf_counter() - t0)

    # single-request latency through the public API (one request's rows as one batch)
    first = [i for i, r in enumerate(wl.request_of) if r == 0]
    one = pack_rows([wl.rows[i] for i in first], [wl.positions[i] for i in first])
    lat = []
    for _ in range(max(5, args.warmup)):
        ts = time.perf_counter()
        backend.score_packed(*one)
        lat.append(time.perf_counter() - ts)

    # Whole-job totals: the pool every rank scored a share of.
    reqs = req_pool.n_requests
    toks_all = req_pool.n_tokens
    rows_all = len(req_pool.rows)
    value = reqs * args.steps / dev_total_s
    pk = peaks()
    gemm_ms, gemm_flops, _gemm_bytes, gemm_n = prof["gemm"]
    achieved = (gemm_flops / 1e12) / (gemm_ms / 1e3) if gemm_ms > 0 else None
    # DRAM traffic of the GEMM class is not measured live (ncu counters come
    # from small-case captures of single launches, profiles/gemm_split_*.md).
    traffic = None
    total_prof_ms = sum(v[0] for v in prof.values())
    line = {
        "metric": "scored requests/s", "value": value, "unit": "requests/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * dev_total_s / args.steps,
        "higher_is_better": True, "scaling": "strong" if strong else "weak", "vs_baseline": None, "dtype": {"fp32": "f32", "q8_0-fp32": "q8_0 x f32", "q4_0-fp32": "q4_0 x f32"}.get(dtype, "bf16"),
        "data": "synthetic",
        "prompt_tokens_per_s": toks_all * args.steps / dev_total_s,
        "questions_per_s": rows_all * args.steps / dev_total_s,
        "p50_request_latency_ms": statistics.median(step_ms),
        "latency_ms": latency_summary(step_ms),
        "p50_single_request_latency_ms": 1000.0 * statistics.median(lat),
        "step_ms": [round(x, 3) for x in step_ms],
        "config": {"workload": WORKLOADS[args.config].format(n=wl.n_requests, dtype=dtype)
                   + ("; prefix cache: each request's shared prefix prefilled once, questions scored as its "
                      "branches" if fork_plan is not None else ""), "model": name,
                   "rows_per_step": rows_all, "requests_per_step": reqs,
                   "tokens_per_step": toks_all, "native_batches_per_step": len(groups),
                   "replicas_per_gpu": n_rep,
                   "l2": "flushed between steps (256 MiB write, outside the timed events); weights 1 GB > L2",
                   "parallelism": f"replicas x{world}",
                   "sharding": ("one pool of {} requests (seed {}) split by shard_by_tokens; this rank: {} requests, "
                                "{} tokens".format(reqs, args.seed, wl.n_requests, n_tok)),
                   **({"timing": "host clock around the synchronous native calls (prefill, branch scoring, "
                                 "release); inputs uploaded inside them", "prefill_tokens_per_step":
                       sum(len(p) for p in fork_plan[0]) * world,
                       "suffix_tokens_per_step": sum(int(a[1][-1]) for _, a in fork_plan[2]) * world}
                      if fork_plan is not None else {})},
        "e2e": {"value": reqs * args.steps / e2e_total_s, "unit": "requests/s", "h2d_bytes_per_step": h2d,
                "d2h_bytes_per_step": d2h,
                "includes": ("hk_score_cached branches (H2D inputs, forward, D2H logits) + host calibration and "
                             "answers" if fork_plan is not None else
                             "hk_score_answers (H2D inputs and question types, forward, on-device calibration and "
                             "answer fields, D2H probabilities and answers; one host thread per replica) + "
                             "answer dicts")},
        "gpu_launches": int(launches),
        "roofline": {"kernel": kernel_label("gemm", dtype)[0],
                     "bound": "tensor", "achieved": achieved,
                     "peak": pk["bf16_tflops_sustained"], "unit": "TFLOP/s",
                     "frac": (achieved / pk["bf16_tflops_sustained"]) if achieved else None,
                     "traffic": traffic,
                     "traffic_note": "per-launch DRAM bytes of single GEMM launches on a small case are in "
                                     "profiles/gemm_split_projections_cfg2_small.md",
                     "work": "algorithmic 2 M N K per projection; split-precision launches also run the 8-bit "
                             "low-part MMAs (half the fp16 MMA time), which are not counted",
                     "peak_source": pk["source"] + " (sustained: kernels timed inside a step)",
                     "launches": int(gemm_n),
                     "timed_over": ("a serial pass of the same steps after the timed region (one handle, one "
                                    "stream; the timed region runs replicas on concurrent streams)"
                                    if serial_ms else "the timed region")},
        **({"serial_pass": {"ms_per_step": statistics.mean(serial_ms),
                            "requests_per_s_this_gpu": wl.n_requests * len(serial_ms) / (sum(serial_ms) / 1000.0),
                            "note": "the same steps with the native batches in sequence on one handle"}}
           if serial_ms else {}),
        "time_shares": {k: round(v[0] / total_prof_ms, 4) for k, v in prof.items() if v[3]}
        if total_prof_ms else {},
        "roofline_per_kernel": kernel_rooflines(prof, pk, dtype),
    }
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        order = [i for r in range(wl.n_requests) for i in range(len(wl.rows)) if wl.request_of[i] == r]
        line["cpu_baseline"] = cpu_baseline(d, dtype, wl, order, prefix_cache=fork_plan is not None)
    line["clocks"] = clk.summary()
    if rank == 0:
        print(json.dumps(line), flush=True)
    if pool is not None:
        pool.shutdown()
    for b in backends[1:]:
        b.close()
    backend.close()
    if world > 1:
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
