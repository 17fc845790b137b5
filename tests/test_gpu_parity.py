"""End-to-end parity of the B200 Kev forward through the C ABI.

Gates:
  * reference golden (tiny_kev, upstream PyTorch): fp32 raw logits < 2e-4 and
    probabilities < 2e-5; bf16 probabilities < 2e-3 -- the gates of
    crates/huncho-backend/tests/kev_reference.rs:64-76 (its half-precision
    gate is 2e-3);
  * the CPU oracle on seeded synthetic models: fp32 probabilities < 1e-4,
    bf16 / int8-weight probabilities < 2e-3 against the fp32 oracle on the
    same (dequantized) weights, and the same argmax on every row;
  * batch invariants of crates/huncho-backend/tests/padded_batch.rs:25-83 and
    native_batch.rs (batched == independent within 1e-4, same argmax).
"""
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from oracle import kev_oracle as ko
from huncho_b200 import calibration, synth
from huncho_b200.backend import pack_rows

from conftest import GOLDEN


def _gpu():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.fixture(scope="module")
def golden():
    return json.loads((GOLDEN / "golden.json").read_text())


def _backend(path, dtype, max_context=512):
    _gpu()
    from huncho_b200.backend import KevBackend
    return KevBackend(path, device=0, dtype=dtype, max_context=max_context)


@pytest.fixture(scope="module")
def tiny_fp32(native_lib):
    return _backend(GOLDEN, "fp32")


def test_tiny_fp32_matches_upstream(tiny_fp32, golden):
    from huncho_b200.backend import ForwardInput
    b = tiny_fp32
    assert b.capabilities().families == ["F2"]
    assert abs(b.temperature - 2.40605) < 1e-5
    for case in golden["cases"]:
        for row in case["rows"]:
            out = b.forward(ForwardInput(row["tokens"], row["positions"]))
            assert out.values.shape == (len(row["positions"]), 1)
            raw = out.values[:, 0]
            assert np.abs(raw - np.array(row["raw_logits"], np.float32)).max() < 2e-4
            p = calibration.calibrate(raw, b.temperature)
            assert np.abs(p - np.array(row["probabilities"], np.float32)).max() < 2e-5
    out = b.forward(ForwardInput([1, 2], [0]))
    assert np.isfinite(out.values).all()
    assert abs(out.values[0, 0] - golden["short_logits"][0]) < 2e-4


@pytest.mark.parametrize("dtype", ["bf16", "fp16"])
def test_tiny_half_matches_upstream_at_half_precision_gate(native_lib, golden, dtype):
    """The reference's own half-precision gate (kev_reference.rs:74-76): 2e-3."""
    from huncho_b200.backend import ForwardInput
    b = _backend(GOLDEN, dtype)
    for case in golden["cases"]:
        for row in case["rows"]:
            raw = b.forward(ForwardInput(row["tokens"], row["positions"])).values[:, 0]
            p = calibration.calibrate(raw, b.temperature)
            assert np.abs(p - np.array(row["probabilities"], np.float32)).max() < 2e-3


def _padded_inputs():
    from huncho_b200.backend import ForwardInput
    return [ForwardInput([(i * 19 + row * 7 + 1) % 380 for i in range(n)], [n - 1, 1, n - 1])
            for row, n in enumerate([5, 13, 47])]


@pytest.mark.parametrize("dtype", ["fp32", "bf16"])
def test_padded_batch_invariants(native_lib, dtype):
    """padded_batch.rs:25-83 on the B200 backend."""
    from huncho_b200.backend import ForwardInput
    from huncho_b200.errors import BackendError
    b = _backend(GOLDEN, dtype)
    inputs = _padded_inputs()
    reference = [b.forward(i) for i in inputs]
    padded = b.forward_padded_batch(inputs)
    for a, r in zip(padded, reference):
        assert a.positions == r.positions
        pa = calibration.calibrate(a.values[:, 0], 2.40605)
        pr = calibration.calibrate(r.values[:, 0], 2.40605)
        assert calibration.argmax(pa.tolist()) == calibration.argmax(pr.tolist())
        assert np.all(np.abs(pa - pr) <= 1e-4)
    wrong = ForwardInput(list(inputs[0].tokens) + [0] * 42, inputs[0].positions)
    w = b.forward(wrong)
    assert np.any(np.abs(w.values - padded[0].values) > 1e-4), "must detect a padded decision row"
    replica = b.replica()
    replay = replica.forward_padded_batch(inputs)
    assert all(np.array_equal(x.values, y.values) for x, y in zip(padded, replay))
    with pytest.raises(BackendError):
        b.forward_batch(inputs)  # unequal lengths
    bad = list(inputs)
    bad[0] = ForwardInput(inputs[0].tokens, [5])
    with pytest.raises(BackendError):
        b.forward_padded_batch(bad)
    with pytest.raises(BackendError):
        b.forward_padded_batch([ForwardInput([], [])])
    with pytest.raises(BackendError):
        b.forward_padded_batch([inputs[0]] * 65)
    assert np.array_equal(reference[0].values, b.forward(inputs[0]).values)


def test_forward_validation_errors(tiny_fp32):
    from huncho_b200.backend import ForwardInput
    from huncho_b200.errors import BackendError, UnsupportedError
    b = tiny_fp32
    with pytest.raises(BackendError):
        b.forward(ForwardInput([1, 2, 384], [0]))  # token >= vocab
    with pytest.raises(BackendError):
        b.forward(ForwardInput([1, 2, 3], [3]))  # position outside
    with pytest.raises(BackendError):
        b.forward(ForwardInput(list(range(1, 300)) * 2, [0]))  # > max_context 512
    with pytest.raises(UnsupportedError):
        b.forward(ForwardInput([1, 2], [0], retain_cache=True))
    assert b.forward(ForwardInput([1, 2, 3], [])).values.shape == (0, 1)
    # The backend stays usable after errors.
    assert np.isfinite(b.forward(ForwardInput([1, 2, 3], [0, 2])).values).all()


def test_equal_length_batch_equals_independent(tiny_fp32):
    from huncho_b200.backend import ForwardInput
    rng = np.random.default_rng(0)
    inputs = [ForwardInput(rng.integers(0, 384, 21).tolist(), [3, 9, 20]) for _ in range(64)]
    batched = tiny_fp32.forward_batch(inputs)
    for inp, out in zip(inputs[:8], batched[:8]):
        single = tiny_fp32.forward(inp)
        assert np.abs(single.values - out.values).max() <= 1e-6


def _synth(synth_root, name, store):
    return synth.write_model(synth_root / f"{name}-{store}", name=name, seed=0, store=store)


@pytest.mark.parametrize("name,dtype,store,tol", [
    ("kev-mini", "fp32", "fp32", 1e-4),
    ("kev-mini", "bf16", "bf16", 2e-3),
    ("kev-mini", "int8w", "bf16", 2e-3),
    ("kev-0.8b-l4", "bf16", "bf16", 2e-3),
    ("kev-0.8b-l4", "int8w", "bf16", 2e-3),
    ("kev-0.8b-l4", "fp16", "bf16", 2e-3),
])
def test_synthetic_model_vs_oracle(native_lib, synth_root, name, dtype, store, tol):
    d = _synth(synth_root, name, store)
    b = _backend(d, dtype, max_context=4096)
    m = ko.load_model(d, dtype)
    vocab = m.cfg.vocab_size
    wl = synth.make_workload(2, vocab, seed=1, n_requests=4)
    rows, pos = wl.rows, wl.positions
    got = b.score_packed(*pack_rows(rows, pos))
    k = 0
    worst = 0.0
    for r, p in zip(rows, pos):
        raw_ref = ko.score_row(m, r, p)
        pr = ko.calibrate(raw_ref, m.temperature)
        pg = calibration.calibrate(got[k:k + len(p)], m.temperature)
        k += len(p)
        worst = max(worst, float(np.abs(pr - pg).max()))
        assert calibration.argmax(pg.tolist()) == calibration.argmax(pr.tolist()), (pr, pg)
    assert worst < tol, worst


def test_full_kev_08b_bf16_vs_oracle(native_lib, synth_root):
    """The benchmark model itself (24 layers, vocab 248320) on two requests of
    the benchmark workload: probabilities within 2e-3 of the fp32 oracle on the
    same bf16 weights, same argmax on every row."""
    d = synth.write_model(synth.default_dir("kev-0.8b", 0, "bf16"), "kev-0.8b", 0, "bf16")
    b = _backend(d, "bf16", max_context=8192)
    m = ko.load_model(d, "bf16")
    wl = synth.make_workload(2, m.cfg.vocab_size, seed=0, n_requests=2)
    got = b.score_packed(*pack_rows(wl.rows, wl.positions))
    k, worst = 0, 0.0
    for r, p in zip(wl.rows, wl.positions):
        pr = ko.calibrate(ko.score_row(m, r, p), m.temperature)
        pg = calibration.calibrate(got[k:k + len(p)], m.temperature)
        k += len(p)
        worst = max(worst, float(np.abs(pr - pg).max()))
        assert calibration.argmax(pg.tolist()) == calibration.argmax(pr.tolist()), (pr, pg)
    print(f"kev-0.8b bf16 vs fp32 oracle: worst probability error {worst:.3g}")
    assert worst < 2e-3, worst


def test_full_size_batch_invariance(native_lib):
    """At the full benchmark size (96 rows in two native batches of 48), each
    row's logits equal those of the same row scored alone (within 1e-4 in
    probability) -- a size-independent property of packed independent rows."""
    d = synth.write_model(synth.default_dir("kev-0.8b", 0, "bf16"), "kev-0.8b", 0, "bf16")
    b = _backend(d, "bf16", max_context=8192)
    wl = synth.make_workload(2, 248320, seed=0)
    assert len(wl.rows) == 96
    outs = []
    for s in (0, 48):
        outs.append(b.score_packed(*pack_rows(wl.rows[s:s + 48], wl.positions[s:s + 48])))
    got = np.concatenate(outs)
    assert np.isfinite(got).all()
    k = 0
    for i, (r, p) in enumerate(zip(wl.rows, wl.positions)):
        if i % 16 == 0:
            single = b.score_packed(*pack_rows([r], [p]))
            pa = calibration.calibrate(single, b.temperature)
            pb = calibration.calibrate(got[k:k + len(p)], b.temperature)
            assert np.abs(pa - pb).max() <= 1e-4
            assert calibration.argmax(pa.tolist()) == calibration.argmax(pb.tolist())
        k += len(p)


@pytest.mark.parametrize("name,dtype,store", [("tiny", "fp32", None), ("tiny", "bf16", None),
                                              ("kev-mini", "bf16", "bf16"), ("kev-0.8b-l4", "bf16", "bf16")])
def test_paged_kv_equals_flat(native_lib, synth_root, name, dtype, store):
    """16-, 64- and 128-token KV pages in a shuffled block table give the flat
    result bit for bit (the reference's pages-vs-flat parity,
    tests/kv_pages.rs:36-103)."""
    d = GOLDEN if name == "tiny" else _synth(synth_root, name, store)
    b = _backend(d, dtype, max_context=4096)
    vocab = b.vocab_size
    wl = synth.make_workload(2, vocab, seed=3, n_requests=3)
    args = pack_rows(wl.rows, wl.positions)
    flat = b.score_packed(*args)
    b.with_kv_page_tokens(16, shuffle_seed=7)
    paged = b.score_packed(*args)
    assert np.array_equal(flat, paged)
    b.with_kv_page_tokens(64, shuffle_seed=0)
    assert np.array_equal(flat, b.score_packed(*args))
    b.with_kv_page_tokens(128, shuffle_seed=1)  # pages wider than a 64-key tile
    assert np.array_equal(flat, b.score_packed(*args))
    b.with_kv_page_tokens(0)
    assert np.array_equal(flat, b.score_packed(*args))


def test_kv_page_tokens_validation(tiny_fp32):
    from huncho_b200.errors import BackendError
    for bad in (8, 48, 512, -16):
        with pytest.raises(BackendError):
            tiny_fp32.with_kv_page_tokens(bad)


def test_replica_on_the_same_gpu_shares_weights(native_lib, synth_root):
    """Backend::replica keeps one copy of the immutable weights per GPU (the
    reference shares them through Arc clones, qwen3_5.rs:2515-2535): the
    replica reports the source's weight store, allocates far less than the
    weights, replays the source bit for bit, and keeps working after the
    source handle is destroyed."""
    import torch
    d = _synth(synth_root, "kev-0.8b-l4", "bf16")
    b = _backend(d, "bf16", max_context=4096)
    wl = synth.make_workload(2, b.vocab_size, seed=4, n_requests=3)
    args = pack_rows(wl.rows, wl.positions)
    ref = b.score_packed(*args)
    nbytes, sid = b.weight_store()
    assert nbytes > 50_000_000
    torch.cuda.synchronize()
    free0, _ = torch.cuda.mem_get_info()
    r = b.replica()
    free1, _ = torch.cuda.mem_get_info()
    assert r.weight_store() == (nbytes, sid)
    assert free0 - free1 < nbytes // 4, (free0 - free1, nbytes)
    b.close()
    assert np.array_equal(r.score_packed(*args), ref)
    r2 = r.replica()
    assert r2.weight_store()[1] == sid
    r.close()
    assert np.array_equal(r2.score_packed(*args), ref)
    r2.close()


def test_int8_weights_take_half_the_projection_bytes(native_lib, synth_root):
    """The int8 per-channel model keeps its projections as int8 in device
    memory (plus fp32 per-row scales): on the 0.8B-layout model, whose
    projections dominate its weights, the store is little more than half of
    the bf16 model's, and both score the same rows within the half-precision
    gate of each other."""
    d = _synth(synth_root, "kev-0.8b-l4", "bf16")
    h16 = _backend(d, "bf16", max_context=4096)
    h8 = _backend(d, "int8w", max_context=4096)
    b16, b8 = h16.weight_store()[0], h8.weight_store()[0]
    assert b8 < 0.56 * b16, (b8, b16)
    wl = synth.make_workload(2, h16.vocab_size, seed=5, n_requests=2)
    args = pack_rows(wl.rows, wl.positions)
    p16 = calibration.calibrate(h16.score_packed(*args), h16.temperature)
    p8 = calibration.calibrate(h8.score_packed(*args), h8.temperature)
    assert np.isfinite(p8).all() and np.abs(p16 - p8).max() < 2e-2
