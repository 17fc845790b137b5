"""Pin the CPU oracle to the reference's golden vectors.

tests/golden/tiny_kev is the reference fixture (crates/huncho-backend/tests/
fixtures/tiny_kev, produced by upstream PyTorch); the gates are those of
crates/huncho-backend/tests/kev_reference.rs:64-76: fp32 raw logits < 2e-4,
fp32 probabilities < 2e-5, and the 2-token `short_logits` row < 2e-4.
"""
import json

import numpy as np
import pytest

from oracle import kev_oracle as ko
from huncho_b200 import calibration, engine

from conftest import GOLDEN


@pytest.fixture(scope="module")
def golden():
    return json.loads((GOLDEN / "golden.json").read_text())


@pytest.fixture(scope="module")
def model():
    return ko.load_model(GOLDEN, "fp32")


def test_metadata(model):
    assert model.meta["base"] == "fixture/qwen3.5"
    assert model.meta["base_revision"] == "1" * 40
    assert abs(model.temperature - 2.40605) < 1e-5
    assert model.head_dim == 4
    assert model.cfg.rotary_dim() == 2  # rope_parameters.partial_rotary_factor 0.5 wins over 0.25


def test_oracle_matches_upstream_logits_and_probabilities(model, golden):
    for case in golden["cases"]:
        for row in case["rows"]:
            raw = ko.score_row(model, row["tokens"], row["positions"])
            assert np.abs(raw - np.array(row["raw_logits"], np.float32)).max() < 2e-4
            p = ko.calibrate(raw, model.temperature)
            assert np.abs(p - np.array(row["probabilities"], np.float32)).max() < 2e-5


def test_short_row_causal_conv(model, golden):
    raw = ko.score_row(model, [1, 2], [0])
    assert np.isfinite(raw).all()
    assert abs(raw[0] - golden["short_logits"][0]) < 2e-4


def test_oracle_calibration_equals_host_calibration(model, golden):
    for case in golden["cases"]:
        for row in case["rows"]:
            raw = np.array(row["raw_logits"], np.float32)
            assert np.array_equal(ko.calibrate(raw, model.temperature),
                                  calibration.calibrate(raw, model.temperature))


def _answers(case, temperature, probs_rows):
    qs = list(case["questions"].items())
    out = {}
    for (name, q), row, probs in zip(qs, case["rows"], probs_rows):
        ans = case["answers"][name]
        if q["type"] == "choice":
            question = engine.Question("choice", labels=list(ans["probabilities"].keys()))
        elif q["type"] == "score":
            question = engine.Question("score", descriptions=list(ans["legend"].values()))
        else:
            question = engine.Question("noul")
        cands = engine.candidates_for(question, row["positions"])
        out[name] = engine.build_answer(question, cands, probs)
    return out


def test_answers_match_upstream_wire_answers(golden):
    """Engine::build_answer on the golden probabilities reproduces the upstream
    wire answers (rounded to 4 decimals by the upstream API)."""
    for case in golden["cases"]:
        probs = [row["probabilities"] for row in case["rows"]]
        got = _answers(case, 2.40605, probs)
        for name, want in case["answers"].items():
            g = got[name]
            assert g["type"] == want["type"]
            if want["type"] == "choice":
                assert g["choice"] == want["choice"]
                assert abs(g["confidence"] - want["confidence"]) < 1e-4
                for k, v in want["probabilities"].items():
                    assert abs(g["probabilities"][k] - v) < 1e-4
            elif want["type"] == "score":
                assert abs(g["score"] - want["score"]) < 1e-4
                assert abs(g["confidence"] - want["confidence"]) < 1e-4
                assert g["legend"] == want["legend"]
            else:
                assert abs(g["noul"] - want["noul"]) < 1e-4


def test_oracle_rejects_bad_rows(model):
    with pytest.raises(ValueError):
        ko.score_row(model, [1, 2, 3], [3])
    with pytest.raises(ValueError):
        ko.score_row(model, [1, 2, 10_000], [0])
    assert ko.score_row(model, [1, 2, 3], []).shape == (0,)


def test_oracle_recurrence_matches_plain_loop():
    """The C recurrence equals a direct Python transcription of
    qwen3_5.rs:965-985 (same fp32 order), bit for bit."""
    rng = np.random.default_rng(3)
    H, T, dk, dv = 2, 5, 4, 3
    q = rng.standard_normal((H, T, dk), dtype=np.float32)
    k = rng.standard_normal((H, T, dk), dtype=np.float32)
    v = rng.standard_normal((H, T, dv), dtype=np.float32)
    g = -rng.random((H, T), dtype=np.float32)
    b = rng.random((H, T), dtype=np.float32)
    out, state = ko.delta_recurrent(q, k, v, g, b)
    f = np.float32
    for h in range(H):
        S = np.zeros((dk, dv), f)
        for t in range(T):
            d = f(np.exp(g[h, t]))
            m = np.zeros(dv, f)
            for i in range(dk):
                for j in range(dv):
                    S[i, j] = f(S[i, j] * d)
                    m[j] = f(m[j] + f(S[i, j] * k[h, t, i]))
            delta = np.array([f(f(v[h, t, j] - m[j]) * b[h, t]) for j in range(dv)], f)
            o = np.zeros(dv, f)
            for i in range(dk):
                for j in range(dv):
                    S[i, j] = f(S[i, j] + f(k[h, t, i] * delta[j]))
                    o[j] = f(o[j] + f(S[i, j] * q[h, t, i]))
            assert np.array_equal(out[h, t], o)
        assert np.array_equal(state[h], S)


def test_int8_quantization_roundtrip():
    rng = np.random.default_rng(0)
    w = rng.standard_normal((8, 64), dtype=np.float32) * np.float32(0.02)
    w[3] = 0
    q, s = ko.quantize_int8_per_channel(w)
    assert q.dtype == np.int8 and s.dtype == np.float32
    assert np.abs(q).max() <= 127
    assert s[3] == 1.0
    deq = q.astype(np.float32) * s[:, None]
    assert np.all(np.abs(deq - w) <= s[:, None] / 2 + 1e-9)


def test_oracle_prefix_cache_matches_full_rows(model, golden):
    """The oracle's prefill / fork / continuation (the CPU side of the GPU fork
    tests): prefixes of 1, 2 and the shared length, continued in chunks of 1, 3
    and all at once, give the full row's logits (prefix_cache.rs:141-205) and
    the upstream golden within its fp32 gate."""
    for case in golden["cases"]:
        rows = case["rows"]
        first = rows[0]["tokens"]
        for prefix_len in (1, 2, rows[0]["prefix_len"]):
            parent = ko.prefill(model, first[:prefix_len])
            assert parent["tokens"] == prefix_len
            for row in rows:
                tokens, positions = row["tokens"], row["positions"]
                full = ko.score_row(model, tokens, positions)
                for chunk in (1, 3, None):
                    branch = ko.copy_cache(parent)
                    offset = prefix_len
                    while offset < positions[0]:
                        end = positions[0] if chunk is None else min(offset + chunk, positions[0])
                        ko.forward_hidden(model, tokens[offset:end], branch)
                        offset = end
                    got = ko.score_branch(model, branch, tokens[offset:], [p - offset for p in positions])
                    assert np.abs(got - full).max() < 1e-5, (got, full)
                    assert np.abs(got - np.asarray(row["raw_logits"], np.float32)).max() < 2e-4
            assert parent["tokens"] == prefix_len  # branches never touch the parent
