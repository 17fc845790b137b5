"""The reference's packed profile on the CPU side: GGML Q8_0 / Q4_0 block
quantization (hand-computed known answers from the published definitions),
the GGUF container, the converter (qwen_quantized.rs:91-208, checked as its
own tests check it: tests/quantized_kev.rs:19-40), and the oracle's packed
forward (activations quantized to Q8_0, per-block integer dots).

No reference execution of the packed path exists here (Rust is absent), so the
block arithmetic is pinned by the known answers below, not by golden vectors.
"""
import json

import numpy as np
import pytest

from huncho_b200 import gguf, quantize

from conftest import GOLDEN

F32 = np.float32


def test_q8_0_block_known_answers():
    x = np.zeros((1, 32), F32)
    x[0, :5] = [1.0, -2.0, 0.5, 0.25, 2.0 / 127 * 0.5]
    d, q = quantize.quantize_q8_0(x)
    # amax 2 -> d = 2/127, 1/d = 63.5: 1 -> 63.5 -> 64 (half away from zero),
    # -2 -> -127, 0.5 -> 31.75 -> 32, 0.25 -> 15.875 -> 16, 1/127 -> 0.5 -> 1.
    assert np.float32(d[0, 0]) == np.float16(F32(2.0) / F32(127.0))
    assert q[0, 0, :5].tolist() == [64, -127, 32, 16, 1]
    assert not q[0, 0, 5:].any()
    d0, q0 = quantize.quantize_q8_0(np.zeros((2, 64), F32))  # zero blocks: d = 0, q = 0
    assert not d0.any() and not q0.any()
    back = quantize.dequantize_q8_0(d, q)
    assert abs(back[0, 1] - (-127 * float(np.float16(2 / 127)))) < 1e-7


def test_q4_0_block_known_answers():
    x = np.zeros((1, 32), F32)
    x[0, :4] = [1.5, -3.0, 3.0, 0.1]
    d, nib = quantize.quantize_q4_0(x)
    # The first value of largest |x| is -3: d = -3 / -8 = 0.375, 1/d = 8/3.
    # 1.5 -> 4 + 8.5 -> 12; -3 -> 0.5 -> 0; 3 -> 16.5 -> min(15, 16) = 15;
    # 0.1 -> 8.7667 -> 8; zeros -> 8.5 -> 8.
    assert float(d[0, 0]) == 0.375
    vals = quantize.q4_values(nib)[0, 0] + 8
    assert vals[:4].tolist() == [12, 0, 15, 8]
    assert (vals[4:] == 8).all()
    assert nib[0, 0, 0] == 12 | (8 << 4)  # value 0 low nibble, value 16 high nibble
    back = quantize.dequantize_q4_0(d, nib)
    assert back[0, :4].tolist() == [1.5, -3.0, 2.625, 0.0]


def test_gguf_round_trip(tmp_path):
    rng = np.random.default_rng(0)
    w = rng.standard_normal((5, 64)).astype(F32)
    dense = rng.standard_normal((3, 7)).astype(F32)
    tensors = {
        "a.q8": (gguf.TYPE_Q8_0, (5, 64), quantize.pack(gguf.TYPE_Q8_0, *quantize.quantize_q8_0(w))),
        "b.q4": (gguf.TYPE_Q4_0, (5, 64), quantize.pack(gguf.TYPE_Q4_0, *quantize.quantize_q4_0(w))),
        "c.f32": (gguf.TYPE_F32, (3, 7), dense.tobytes()),
    }
    meta = {"general.architecture": "huncho-kev-qwen3.5", "huncho.config_json": "{}", "n": 7}
    gguf.write(tmp_path / "t.gguf", meta, tensors)
    m2, t2 = gguf.read(tmp_path / "t.gguf")
    assert m2 == meta
    assert set(t2) == set(tensors)
    for k, (t, shape, raw) in tensors.items():
        assert t2[k][0] == t and t2[k][1] == shape and bytes(t2[k][2]) == raw
    d, q = quantize.unpack(gguf.TYPE_Q8_0, t2["a.q8"][2], 5, 64)
    d_ref, q_ref = quantize.quantize_q8_0(w)
    assert (d == d_ref).all() and (q == q_ref).all()
    with pytest.raises(ValueError):
        gguf.write(tmp_path / "bad.gguf", {}, {"x": (gguf.TYPE_Q8_0, (1, 33), b"")})


@pytest.mark.parametrize("scheme", ["q8_0-fp32", "q4_0-fp32"])
def test_converter_on_the_tiny_package(tmp_path, scheme):
    pkg = quantize.write_package(GOLDEN, scheme, tmp_path / scheme)
    stats = json.loads((pkg / "quantization.json").read_text())
    assert stats["projection_count"] == 15
    assert stats["packed_projection_bytes"] < stats["source_projection_bytes"]
    assert stats["dense_backbone_bytes"] > 0
    meta, tensors = gguf.read(pkg / "backbone.gguf")
    assert meta["huncho.quantization"] == quantize.PROFILES[scheme]
    widths = json.loads(meta["huncho.input_widths"])
    assert len(widths) == 15 and all(v == 16 or v == 32 for v in widths.values())
    packed = [n for n, (t, _, _) in tensors.items() if t != gguf.TYPE_F32]
    assert sorted(packed) == sorted(widths)
    assert all(tensors[n][1][1] % 32 == 0 for n in packed)  # rows padded to 32 inputs


@pytest.mark.parametrize("scheme", ["q8_0-fp32", "q4_0-fp32"])
def test_packed_oracle_forward(tmp_path, scheme):
    from oracle import kev_oracle as ko
    pkg = quantize.write_package(GOLDEN, scheme, tmp_path / scheme)
    mq = ko.load_model(pkg, scheme)
    mf = ko.load_model(GOLDEN, "fp32")
    with pytest.raises(ValueError):  # the artifact's profile must match
        ko.load_model(pkg, "q4_0-fp32" if scheme == "q8_0-fp32" else "q8_0-fp32")
    golden = json.loads((GOLDEN / "golden.json").read_text())
    changed = False
    for case in golden["cases"]:
        for row in case["rows"]:
            lq = ko.score_row(mq, row["tokens"], row["positions"])
            lf = ko.score_row(mf, row["tokens"], row["positions"])
            p = ko.calibrate(lq, 2.40605)
            assert np.all(np.isfinite(p)) and abs(float(p.sum()) - 1.0) <= 1e-5
            changed |= not np.array_equal(lq, lf)
            # Weight + activation quantization moves the logits a little.
            assert np.abs(lq - lf).max() < (0.05 if scheme == "q8_0-fp32" else 0.5)
    assert changed


def test_packed_linear_matches_block_definition():
    """The oracle's packed matmul against an independent per-element loop."""
    from oracle import kev_oracle as ko
    rng = np.random.default_rng(1)
    w = rng.standard_normal((3, 40)).astype(F32)
    wp = np.concatenate([w, np.zeros((3, 24), F32)], axis=1)
    d, q = quantize.quantize_q8_0(wp)
    pw = ko.PackedWeight(q=q, d=d.astype(F32), width=40)
    x = rng.standard_normal((2, 40)).astype(F32)
    got = ko.packed_linear(x, pw)
    xp = np.concatenate([x, np.zeros((2, 24), F32)], axis=1)
    dx, qx = quantize.quantize_q8_0(xp)
    for m in range(2):
        for n in range(3):
            acc = F32(0.0)
            for b in range(2):
                s = int(sum(int(qx[m, b, i]) * int(q[n, b, i]) for i in range(32)))
                acc = F32(acc + F32(F32(F32(s) * F32(d[n, b])) * F32(dx[m, b])))
            assert got[m, n] == acc
