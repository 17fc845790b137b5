"""The `/v1/systemone` answer semantics above the backend (huncho-core engine.rs).

A Kev question is one row: its candidates are the option readout positions
(the `<box_end>` tokens, crates/huncho-core/src/prompt/kev.rs:92-192) and the
decision row is the row's last token. This module turns a backend's raw
pointer logits into calibrated probabilities and typed answers exactly as
Engine::build_answer does (engine.rs:1448-1513), and batches rows into
groups of at most `BatchLimits.max_rows` (batching.rs:21-80).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import calibration
from .backend import ForwardInput
from .errors import CalibrationError


@dataclass
class Question:
    """A typed question: `choice` (labels), `noul` (yes/no) or `score` (levels)."""
    type: str
    labels: list = field(default_factory=list)        # choice labels in option order
    descriptions: list = field(default_factory=list)  # score legend, per level

    def n_options(self) -> int:
        if self.type == "noul":
            return 2
        return len(self.labels) if self.type == "choice" else len(self.descriptions)


@dataclass
class Candidate:
    label: str
    index: int
    position: int
    description: Optional[str] = None


def candidates_for(q: Question, positions: Sequence[int]) -> list:
    """Candidate labels in Kev's option order; noul is [no, yes] (prompt/kev.rs:139-158)."""
    if q.type == "noul":
        labels = ["no", "yes"]
    elif q.type == "choice":
        labels = list(q.labels)
    elif q.type == "score":
        labels = [str(i) for i in range(len(q.descriptions))]
    else:
        raise ValueError(f"unknown question type {q.type}")
    if len(labels) != len(positions):
        raise ValueError("one readout position per candidate is required")
    desc = q.descriptions if q.type == "score" else [None] * len(labels)
    return [Candidate(label=l, index=i, position=int(p), description=desc[i])
            for i, (l, p) in enumerate(zip(labels, positions))]


def build_answer(q: Question, candidates: Sequence[Candidate], probabilities, kev: bool = True) -> dict:
    """Engine::build_answer (engine.rs:1448-1513) with Kev's score confidence."""
    p = np.asarray(probabilities, dtype=np.float32)
    if len(candidates) != p.size:
        raise CalibrationError(f"candidate/probability count mismatch: {len(candidates)} vs {p.size}")
    if kev and q.type == "score":
        conf = calibration.confidence_score(p)
    else:
        conf = calibration.confidence_peak(p)
    if q.type == "choice":
        best = calibration.argmax(p.tolist())
        return {"type": "choice", "choice": candidates[best].label, "confidence": conf,
                "probabilities": {c.label: float(p[c.index]) for c in candidates}}
    if q.type == "score":
        score = np.float32(0.0)
        for c in candidates:
            score = np.float32(score + np.float32(c.index) * p[c.index])
        return {"type": "score", "score": float(score), "confidence": conf,
                "legend": {c.label: (c.description or "") for c in candidates},
                "probabilities": {c.label: float(p[c.index]) for c in candidates}}
    if q.type == "noul":
        yes = next((i for i, c in enumerate(candidates) if c.label == "yes"), None)
        return {"type": "noul", "noul": float(p[yes]) if yes is not None else 0.0}
    raise ValueError(f"unknown question type {q.type}")


def score_rows(backend, rows: Sequence[Sequence[int]], positions: Sequence[Sequence[int]],
               temperature: Optional[float] = None) -> list:
    """Raw logits and calibrated probabilities of independent question rows.

    Rows go to the backend in groups of at most `batch_limits().max_rows`
    (the engine's padded groups, batching.rs:33-80); every row is calibrated
    with the package temperature (cal:186-196).
    """
    t = backend.temperature if temperature is None else temperature
    limit = backend.batch_limits().max_rows
    out = []
    for s in range(0, len(rows), limit):
        group = [ForwardInput(tokens=r, positions=p) for r, p in zip(rows[s:s + limit], positions[s:s + limit])]
        for o in backend.forward_padded_batch(group):
            raw = o.values[:, 0]
            out.append((raw, calibration.calibrate(raw, t)))
    return out


def answer_from_record(q: Question, candidates: Sequence[Candidate], probabilities, record) -> dict:
    """The build_answer dict from a device answer record (hk_answer: best,
    status, confidence, value) and the device probabilities."""
    if int(record["status"]) != 0:
        raise CalibrationError("temperature scaling produced nonfinite probabilities"
                               if int(record["status"]) == 2 else "logits must be finite")
    p = np.asarray(probabilities, dtype=np.float32)
    if len(candidates) != p.size:
        raise CalibrationError(f"candidate/probability count mismatch: {len(candidates)} vs {p.size}")
    conf, value, best = float(record["confidence"]), float(record["value"]), int(record["best"])
    if q.type == "choice":
        return {"type": "choice", "choice": candidates[best].label, "confidence": conf,
                "probabilities": {c.label: float(p[c.index]) for c in candidates}}
    if q.type == "score":
        return {"type": "score", "score": value, "confidence": conf,
                "legend": {c.label: (c.description or "") for c in candidates},
                "probabilities": {c.label: float(p[c.index]) for c in candidates}}
    if q.type == "noul":
        return {"type": "noul", "noul": value}
    raise ValueError(f"unknown question type {q.type}")


def score_questions(backend, rows: Sequence[Sequence[int]], positions: Sequence[Sequence[int]],
                    questions: Sequence[Question], temperature: Optional[float] = None) -> list:
    """Answers of independent question rows, calibrated on the device.

    The same answers as score_rows + build_answer (calibration.rs:36-64,
    87-147; engine.rs:1448-1513), computed for each group of at most
    `batch_limits().max_rows` rows by one hk_score_answers call.
    """
    from .backend import pack_rows
    limit = backend.batch_limits().max_rows
    out = []
    for s in range(0, len(rows), limit):
        rs, ps, qs = rows[s:s + limit], positions[s:s + limit], questions[s:s + limit]
        probs, rec = backend.score_answers(*pack_rows(rs, ps), [q.type for q in qs], temperature=temperature)
        k = 0
        for q, pos, r in zip(qs, ps, rec):
            n = len(pos)
            out.append(answer_from_record(q, candidates_for(q, pos), probs[k:k + n], r))
            k += n
    return out
