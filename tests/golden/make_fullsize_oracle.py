"""Generate the full-size oracle fixtures under tests/golden/fullsize/.

Each fixture holds the CPU oracle's raw pointer logits for question rows of one
benchmark configuration, on the seeded synthetic model of that configuration
(huncho_b200.synth; same seeds as bench.py and the GPU tests). The oracle at
these sizes takes minutes on a CPU, so it runs once here and the GPU parity
tests (tests/test_gpu_fullsize.py) compare the B200 forward against the stored
logits. Both sides regenerate the model and the rows from their seeds; the
fixture carries fingerprints of both, which the test checks first.

Configurations (the workload definitions of BASELINE.json):
  cfg1  Kev-0.8B fp32 weights, fp32 model, 1 x 256 tokens, choice-4
  cfg2  Kev-0.8B bf16, all 96 question rows of the benchmark workload (seed 0)
  cfg3  Kev-0.8B bf16 weights quantized int8 per output channel, 16 x 1024, choice-8
  cfg4  Kev-0.8B bf16, 4 x 8192 tokens, noul
  cfg5  Kev-4B bf16, 24 requests, lengths log-uniform in [32, 2048], mixed questions

Usage: python tests/golden/make_fullsize_oracle.py [cfg1 cfg2 ...]
"""
from __future__ import annotations

import hashlib
import json
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
if str(ROOT) not in sys.path:
    sys.path.insert(0, str(ROOT))

from huncho_b200 import synth  # noqa: E402

OUT = Path(__file__).resolve().parent / "fullsize"

# name -> (synthetic model, weight store, model dtype, workload cfg, workload seed, n_requests)
CASES = {
    "cfg1": ("kev-0.8b", "fp32", "fp32", 1, 0, None),
    "cfg2": ("kev-0.8b", "bf16", "bf16", 2, 0, None),
    "cfg3": ("kev-0.8b", "bf16", "int8w", 3, 0, 16),
    "cfg4": ("kev-0.8b", "bf16", "bf16", 4, 0, 4),
    "cfg5": ("kev-4b", "bf16", "bf16", 5, 0, 24),
}


def model_fingerprint(model_dir: Path) -> str:
    """sha256 over the safetensors header and the first / last MiB of the data."""
    h = hashlib.sha256()
    for name in ("model.safetensors", "pointer_head.safetensors"):
        p = Path(model_dir) / name
        size = p.stat().st_size
        with open(p, "rb") as f:
            h.update(f.read(1 << 20))
            f.seek(max(0, size - (1 << 20)))
            h.update(f.read(1 << 20))
        h.update(str(size).encode())
    return h.hexdigest()


def rows_fingerprint(rows, positions) -> str:
    h = hashlib.sha256()
    for r, p in zip(rows, positions):
        h.update(np.asarray(r, np.uint32).tobytes())
        h.update(np.asarray(p, np.int32).tobytes())
    return h.hexdigest()


def case_model_dir(name: str) -> Path:
    model, store, _dtype, *_ = CASES[name]
    return synth.write_model(synth.default_dir(model, 0, store), model, 0, store)


def case_workload(name: str, vocab: int):
    _m, _s, _d, cfg, seed, n_req = CASES[name]
    return synth.make_workload(cfg, vocab, seed=seed, n_requests=n_req)


def generate(name: str) -> Path:
    from oracle import kev_oracle as ko
    model, store, dtype, cfg, seed, n_req = CASES[name]
    d = case_model_dir(name)
    m = ko.load_model(d, dtype)
    wl = case_workload(name, m.cfg.vocab_size)
    rows = []
    t0 = time.time()
    for i, (r, p, q) in enumerate(zip(wl.rows, wl.positions, wl.qtypes)):
        raw = ko.score_row(m, r, p)
        rows.append({"len": len(r), "positions": list(map(int, p)), "qtype": q,
                     "raw_logits": [float(v) for v in raw]})
        print(f"{name} row {i + 1}/{len(wl.rows)} ({len(r)} tokens) {time.time() - t0:.0f}s", flush=True)
    OUT.mkdir(exist_ok=True)
    path = OUT / f"{name}.json"
    path.write_text(json.dumps({
        "config": name, "model": model, "store": store, "dtype": dtype, "model_seed": 0,
        "workload_cfg": cfg, "workload_seed": seed, "n_requests": n_req,
        "model_fingerprint": model_fingerprint(d),
        "rows_fingerprint": rows_fingerprint(wl.rows, wl.positions),
        "temperature": m.temperature,
        "oracle": "oracle/kev_oracle.py score_row (fp32 math on the model dtype's weights)",
        "rows": rows}, indent=0))
    return path


if __name__ == "__main__":
    for n in sys.argv[1:] or list(CASES):
        print(generate(n), flush=True)
