"""Host calibration against the reference's bit-exactness sweep
(crates/huncho-core/src/calibration.rs:309-420): for many sizes, logit
patterns (zeros, signed zeros, +-f32::MAX, subnormal steps, tiny and large
ramps, seeded uniforms) and temperatures from the smallest normal float to
f32::MAX, `calibrate` equals, bit for bit, a separate statement of the
original arithmetic: fp32 exponential of (l - max) * (1/T), fp64 sum and
division in input order, fp32 result. Invalid temperatures and logits are
rejected, and the C-library exponential the host uses is the one Rust's
f32::exp calls on Linux.
"""
import ctypes
import math

import numpy as np
import pytest

from huncho_b200 import calibration
from huncho_b200.errors import CalibrationError

F32 = np.float32
F32_MAX = float(np.finfo(F32).max)
F32_MIN_NORMAL = float(np.finfo(F32).tiny)

_libm = ctypes.CDLL("libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]


def _original(logits, temperature):
    """The arithmetic spelled out one value at a time."""
    if not logits:
        return []
    inv_t = F32(1.0) / F32(temperature)
    mx = max(F32(v) for v in logits)
    ex = []
    with np.errstate(over="ignore", invalid="ignore"):
        for v in logits:
            ex.append(float(_libm.expf(float(F32(F32(v) - mx) * inv_t))))
    s = 0.0
    for e in ex:
        s += e
    return [F32(e / s) for e in ex]


def _patterns(size, seed):
    """Logit patterns per size; `seed` is a 64-bit LCG state carried across calls."""
    out = []
    for pattern in range(8):
        vals = []
        for i in range(size):
            seed = (seed * 6364136223846793005 + 1442695040888963407) % (1 << 64)
            if pattern == 0:
                v = 0.0
            elif pattern == 1:
                v = -0.0 if i % 2 == 0 else 0.0
            elif pattern == 2:
                v = F32_MAX if i % 2 == 0 else -F32_MAX
            elif pattern == 3:
                v = float(F32(i - size / 2.0) * F32(F32_MIN_NORMAL))
            elif pattern == 4:
                v = float(F32(i - size / 2.0) * F32(1e-5))
            elif pattern == 5:
                v = float(F32(i - size / 2.0) * F32(100.0))
            else:
                v = float(F32((float(F32(seed >> 32)) / float(F32(2 ** 32 - 1)) - 0.5) * 31.0))
            vals.append(v)
        out.append(vals)
    return out, seed


@pytest.mark.parametrize("size", [0, 1, 2, 3, 5, 10, 11, 63, 64, 127, 256])
def test_calibrate_equals_original_float_bits(size):
    seed = 0x7123ABCD + size
    rows, _ = _patterns(size, seed)
    for logits in rows:
        for t in (F32_MIN_NORMAL, 1e-20, 0.03125, 0.75, 1.0, 2.40605, 1e6, F32_MAX):
            want = np.array(_original(logits, t), dtype=F32)
            got = calibration.calibrate(np.array(logits, F32), t)
            assert got.dtype == F32 and got.shape == want.shape
            assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), (logits[:4], t)


def test_calibrate_rejections():
    logits = np.array([1.0, -2.0, 3.0], F32)
    for t in (0.0, -1.0, float("nan"), float("inf")):
        with pytest.raises(CalibrationError, match="temperature must be positive and finite"):
            calibration.calibrate(logits, t)
    # The smallest subnormal temperature is valid, but 1/T is infinite and
    # (max - max) * inf is NaN: rejected after scaling.
    with pytest.raises(CalibrationError, match="nonfinite probabilities"), np.errstate(all="ignore"):
        calibration.calibrate(logits, float(np.array([1], np.uint32).view(F32)[0]))
    for bad in (float("nan"), float("inf"), float("-inf")):
        with pytest.raises(CalibrationError, match="logits must be finite"):
            calibration.calibrate(np.array([1.0, bad], F32), 1.0)


def test_small_cases_and_host_exponential():
    p = calibration.calibrate(np.array([1.0, 2.0, 3.0], F32), 1.0)
    assert abs(float(p.sum()) - 1.0) < 1e-6 and p[2] > p[1] > p[0]
    p1 = calibration.calibrate(np.array([2.0, 0.0], F32), 1.0)
    p4 = calibration.calibrate(np.array([2.0, 0.0], F32), 4.0)
    assert p1[0] > p4[0]  # a higher temperature flattens
    xs = np.linspace(-30.0, 0.0, 4001).astype(F32)
    host = calibration.expf(xs)
    ref = np.array([_libm.expf(float(v)) for v in xs], F32)
    assert np.array_equal(host, ref)
    # within half an ulp-and-a-bit of the exact exponential
    exact = np.exp(xs.astype(np.float64))
    assert np.all(np.abs(host.astype(np.float64) - exact) <= 0.51 * np.spacing(host).astype(np.float64))
    assert math.isclose(float(calibration.expf(np.array([0.0], F32))[0]), 1.0)


def test_confidence_known_answers():
    """The reference's confidence values (calibration.rs:447-461)."""
    for probs, want, tol in (([0.61, 0.35, 0.04], 0.42, 0.01), ([0.0, 0.57, 0.43], 0.35, 0.01),
                             ([0.0, 0.89, 0.11], 0.84, 0.01), ([0.84, 0.10, 0.06], 0.76, 0.01),
                             ([1.0, 0.0], 1.0, 1e-6), ([0.5, 0.5], 0.0, 1e-6)):
        assert abs(calibration.confidence_peak(probs) - want) < tol
    assert abs(calibration.confidence_entropy([1.0, 0.0]) - 1.0) < 1e-6
    assert abs(calibration.confidence_entropy([0.5, 0.5]) - 0.0) < 1e-6
    assert calibration.argmax([0.2, 0.4, 0.4]) == 1  # first maximum
