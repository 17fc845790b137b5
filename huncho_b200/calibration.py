"""Calibration math of huncho-core (crates/huncho-core/src/calibration.rs).

Temperature softmax keeps the reference's mixed precision exactly: the
exponential of (l - max) * (1/T) is fp32, the sum and the division run in fp64
in input order, and each probability is rounded back to fp32
(calibration.rs:43-64). The fp32 exponential is the C library's `expf`, the
function Rust's `f32::exp` calls on Linux; numpy's own float32 `exp` differs
from it in the last bit for a large share of inputs.
"""
from __future__ import annotations

import ctypes
import ctypes.util
import math

import numpy as np

from .errors import CalibrationError

F32 = np.float32

_libm = ctypes.CDLL(ctypes.util.find_library("m") or "libm.so.6")
_expf = _libm.expf
_expf.restype = ctypes.c_float
_expf.argtypes = [ctypes.c_float]


def expf(x) -> np.ndarray:
    """Elementwise C-library fp32 exponential of a float32 array."""
    return np.array([_expf(v) for v in np.asarray(x, dtype=F32).ravel().tolist()], dtype=F32)


def bucket_size(n_options: int) -> str:
    """calibration.rs:12-22."""
    if n_options <= 2:
        return "2"
    if n_options <= 5:
        return "3-5"
    if n_options <= 10:
        return "6-10"
    return "11+"


def softmax_temperature(logits, temperature) -> np.ndarray:
    """calibration.rs:36-64 (unchecked)."""
    l = np.asarray(logits, dtype=F32)
    if l.size == 0:
        return l.copy()
    inv_t = F32(1.0) / F32(temperature)
    mx = F32(np.max(l))
    with np.errstate(over="ignore", invalid="ignore"):
        e = expf(((l - mx) * inv_t).astype(F32))
    s = 0.0
    for v in e.tolist():
        s += v
    return np.array([v / s for v in e.tolist()], dtype=np.float64).astype(F32)


def softmax(logits) -> np.ndarray:
    return softmax_temperature(logits, 1.0)


def calibrate(logits, temperature) -> np.ndarray:
    """calibration.rs:172-176 with the validation of 198-218."""
    t = F32(temperature)
    if not math.isfinite(float(t)) or t <= 0:
        raise CalibrationError(f"temperature must be positive and finite, got {temperature}")
    l = np.asarray(logits, dtype=F32)
    if not np.all(np.isfinite(l)):
        raise CalibrationError("logits must be finite")
    p = softmax_temperature(l, t)
    if not np.all(np.isfinite(p)):
        raise CalibrationError("temperature scaling produced nonfinite probabilities")
    return p


def argmax(values) -> int:
    """First maximum (calibration.rs:87-95)."""
    best = 0
    for i, v in enumerate(values):
        if v > values[best]:
            best = i
    return best


def confidence_peak(probs) -> float:
    """(p_max - 1/n) / (1 - 1/n), clamped (calibration.rs:114-127)."""
    p = np.asarray(probs, dtype=F32)
    n = p.size
    if n <= 1:
        return float(np.clip(p[0] if n else F32(0.0), 0.0, 1.0))
    uniform = F32(1.0) / F32(n)
    denom = F32(1.0) - uniform
    if denom <= 0:
        return 1.0
    return float(np.clip((F32(np.max(p)) - uniform) / denom, F32(0.0), F32(1.0)))


def confidence_score(probs) -> float:
    """Kev score confidence (calibration.rs:131-147)."""
    p = np.asarray(probs, dtype=F32)
    n = p.size
    if n <= 1:
        return 1.0
    center = F32(n - 1) / F32(2.0)
    uniform_dev = F32(sum(abs(F32(i) - center) for i in range(n))) / F32(n)
    mode = F32(argmax(p.tolist()))
    dev = F32(0.0)
    for i, pi in enumerate(p):
        dev = F32(dev + pi * abs(F32(i) - mode))
    return float(np.clip(F32(1.0) - dev / uniform_dev, F32(0.0), F32(1.0)))


def entropy(probs) -> float:
    h = 0.0
    for p in np.asarray(probs, dtype=F32).tolist():
        if p > 0:
            h += p * math.log2(p)
    return float(F32(-h))


def confidence_entropy(probs) -> float:
    """1 - H(p) / log2(n) (calibration.rs:153-165)."""
    p = np.asarray(probs, dtype=F32)
    n = p.size
    if n <= 1:
        return float(np.clip(p[0] if n else F32(0.0), 0.0, 1.0))
    max_h = F32(math.log2(n))
    if max_h <= 0:
        return 1.0
    return float(np.clip(F32(1.0) - F32(entropy(p)) / max_h, F32(0.0), F32(1.0)))
