"""Full-size parity on every benchmark configuration, through the C ABI.

The CPU oracle at these sizes takes minutes, so its raw pointer logits are
stored once per configuration under tests/golden/fullsize/ by
tests/golden/make_fullsize_oracle.py (which documents the cases). Each test
regenerates the same seeded synthetic model and question rows, checks both
against the fixture's fingerprints, scores every row on the B200 and compares
calibrated probabilities with the oracle's:

  * cfg1 Kev-0.8B fp32, 1 x 256: within 1e-4 (the reference's fp32 gate);
  * cfg2 Kev-0.8B bf16, all 96 benchmark rows; cfg3 int8 per-channel weights,
    16 x 1024 tokens, choice-8; cfg4 4 x 8192 tokens on 16-token pages in a
    shuffled block table; cfg5 Kev-4B bf16, 24 mixed rows: within 2e-3 (the
    reference's half-precision gate, tests/kev_reference.rs:64-76);
  * every configuration: the same argmax as the oracle on every row.

Set HK_PARITY_REPORT to a file path to append each configuration's worst
probability error and row count as one JSON line.
"""
import importlib.util
import json
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from huncho_b200 import calibration
from huncho_b200.backend import pack_rows

from conftest import ROOT

FIXTURES = ROOT / "tests" / "golden" / "fullsize"
TOL = {"cfg1": 1e-4, "cfg2": 2e-3, "cfg3": 2e-3, "cfg4": 2e-3, "cfg5": 2e-3}


def _generator():
    spec = importlib.util.spec_from_file_location("make_fullsize_oracle",
                                                  ROOT / "tests" / "golden" / "make_fullsize_oracle.py")
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _report(entry: dict) -> None:
    path = os.environ.get("HK_PARITY_REPORT")
    if path:
        with open(path, "a") as f:
            f.write(json.dumps(entry) + "\n")


def _case(name):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    fx_path = FIXTURES / f"{name}.json"
    if not fx_path.exists():
        pytest.fail(f"missing fixture {fx_path.name}; run tests/golden/make_fullsize_oracle.py {name}")
    fx = json.loads(fx_path.read_text())
    gen = _generator()
    d = gen.case_model_dir(name)
    assert gen.model_fingerprint(d) == fx["model_fingerprint"], "synthetic model differs from the fixture's"
    vocab = json.loads((d / "config.json").read_text())["vocab_size"]
    wl = gen.case_workload(name, vocab)
    assert gen.rows_fingerprint(wl.rows, wl.positions) == fx["rows_fingerprint"], "rows differ from the fixture's"
    assert len(wl.rows) == len(fx["rows"])
    return fx, d, wl


def _compare(name, fx, got_rows, temperature):
    worst, flips, per_row = 0.0, [], []
    for i, (row, got) in enumerate(zip(fx["rows"], got_rows)):
        pr = calibration.calibrate(np.asarray(row["raw_logits"], np.float32), temperature)
        pg = calibration.calibrate(np.asarray(got, np.float32), temperature)
        per_row.append(float(np.abs(pr - pg).max()))
        worst = max(worst, per_row[-1])
        if calibration.argmax(pg.tolist()) != calibration.argmax(pr.tolist()):
            flips.append(i)
    _report({"config": name, "rows": len(fx["rows"]), "worst_abs_prob_err": worst, "gate": TOL[name],
             "argmax_mismatches": len(flips), "per_row": [round(e, 7) for e in per_row],
             "raw_logits": [[float(v) for v in g] for g in got_rows]})
    print(f"{name}: {len(fx['rows'])} rows, worst |dp| {worst:.3g} (gate {TOL[name]}), argmax flips {flips}")
    assert not flips, f"argmax differs from the oracle on rows {flips}"
    assert worst < TOL[name], worst


def _score(b, wl, batch):
    out = []
    for s in range(0, len(wl.rows), batch):
        rows, pos = wl.rows[s:s + batch], wl.positions[s:s + batch]
        got = b.score_packed(*pack_rows(rows, pos))
        k = 0
        for p in pos:
            out.append(got[k:k + len(p)])
            k += len(p)
    return out


@pytest.mark.parametrize("name", ["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
def test_fullsize_config_vs_oracle(native_lib, name):
    from huncho_b200.backend import KevBackend
    fx, d, wl = _case(name)
    b = KevBackend(d, device=0, dtype=fx["dtype"], max_context=8192)
    try:
        if name == "cfg4":
            b.with_kv_page_tokens(16, shuffle_seed=7)
        got = _score(b, wl, 48 if name == "cfg2" else 64)
        _compare(name, fx, got, b.temperature)
    finally:
        b.close()


def test_fullsize_cfg2_device_answers_vs_oracle(native_lib):
    """The benchmark's end-to-end call (hk_score_answers: forward, then the
    temperature softmax and answers on the device) on all 96 rows against the
    oracle's probabilities, with the answer's choice equal to the oracle's
    argmax."""
    from huncho_b200.backend import KevBackend
    fx, d, wl = _case("cfg2")
    b = KevBackend(d, device=0, dtype="bf16", max_context=8192)
    try:
        worst = 0.0
        for s in range(0, len(wl.rows), 48):
            rows, pos, qt = wl.rows[s:s + 48], wl.positions[s:s + 48], wl.qtypes[s:s + 48]
            probs, ans = b.score_answers(*pack_rows(rows, pos), qt)
            k = 0
            for i, p in enumerate(pos):
                pr = calibration.calibrate(np.asarray(fx["rows"][s + i]["raw_logits"], np.float32), b.temperature)
                worst = max(worst, float(np.abs(probs[k:k + len(p)] - pr).max()))
                if qt[i] == "choice":
                    assert ans["best"][i] == calibration.argmax(pr.tolist())
                k += len(p)
        print(f"cfg2 device answers: worst |dp| {worst:.3g}")
        assert worst < 2e-3, worst
    finally:
        b.close()
