"""The reference's packed profiles (q8_0-fp32 / q4_0-fp32) on the GPU.

* The packed projection kernel (Q8_0 activation quantization + per-block int8
  tcgen05 dots with the block scales applied in the reference's order)
  equals the oracle's block-sequential definition bit for bit, on shapes with
  ragged edges, one row, more tiles than SMs and 112 blocks per row.
* Whole packed packages (converted from the tiny golden package and from a
  synthetic model) against the oracle's packed forward: raw logits within the
  fp32 model's gate, probabilities within the reference's own gate for packed
  execution (1e-4, tests/quantized_kev.rs:10-17; for the deeper synthetic
  model, twice the oracle's own one-ulp sensitivity when that is larger, since
  Q8_0 activation rounding turns a one-ulp input difference into a quantum),
  same argmax; batched,
  duplicated and prefix-forked rows equal independent ones (the isolation
  checks of quantized_kev.rs:85-150); an artifact of the other scheme is
  rejected (quantized_kev.rs:66-76).
"""
import ctypes
import json

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from huncho_b200 import calibration, quantize, synth
from huncho_b200.backend import ForwardInput, pack_rows

from conftest import GOLDEN

F32 = np.float32


def _torch():
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _run_op(lib, x, wq, wd, K, residual=None):
    torch = _torch()
    M, N, kp = x.shape[0], wq.shape[0], wq.shape[1]
    xt = torch.from_numpy(np.ascontiguousarray(x)).cuda()
    wqt = torch.from_numpy(np.ascontiguousarray(wq)).cuda()
    wdt = torch.from_numpy(np.ascontiguousarray(wd, dtype=F32)).cuda()
    xq = torch.empty((M, kp), dtype=torch.int8, device="cuda")
    xd = torch.empty((M, kp // 32), dtype=torch.float32, device="cuda")
    out = (torch.from_numpy(residual.copy()).cuda() if residual is not None
           else torch.full((M, N), float("nan"), device="cuda"))
    lib.hk_op_gemm_packed.argtypes = [ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 5 + \
        [ctypes.c_int, ctypes.c_int, ctypes.c_void_p]
    rc = lib.hk_op_gemm_packed(M, N, K, kp, _p(xt), xt.stride(0), _p(wqt), _p(wdt), _p(xq), _p(xd), _p(out),
                               out.stride(0), 1 if residual is not None else 0, None)
    assert rc == 0
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("scheme", ["q8_0", "q4_0"])
# (2100, 1300, 512): more 128 x 128 tiles than SMs, so CTAs run several tiles
# (the block accumulators carry over between tiles); (700, 1100, 3584): the MLP
# down projection's 112 blocks per row.
@pytest.mark.parametrize("M,N,K", [(300, 130, 200), (1, 1, 1), (129, 65, 64), (64, 3584 // 8, 1024),
                                   (2100, 1300, 512), (700, 1100, 3584)])
def test_packed_gemm_bit_exact_vs_oracle(native_lib, scheme, M, N, K):
    from oracle import kev_oracle as ko
    rng = np.random.default_rng(M + N + K)
    kp = -(-K // 32) * 32
    w = np.zeros((N, kp), F32)
    w[:, :K] = rng.standard_normal((N, K)).astype(F32) * 0.05
    if scheme == "q8_0":
        d, q = quantize.quantize_q8_0(w)
    else:
        d, nib = quantize.quantize_q4_0(w)
        q = quantize.q4_values(nib)
    wq = q.reshape(N, kp).astype(np.int8)
    wd = d.astype(F32)
    x = (rng.standard_normal((M, K)) * rng.uniform(0.1, 4.0, (M, 1))).astype(F32)
    x[:, ::7] = 0.0  # exact zeros and zero blocks
    ref = ko.packed_linear(x, ko.PackedWeight(q=q, d=wd, width=K))
    got = _run_op(native_lib, x, wq, wd, K)
    np.testing.assert_array_equal(got, ref)
    res = rng.standard_normal((M, N)).astype(F32)
    got = _run_op(native_lib, x, wq, wd, K, residual=res)
    np.testing.assert_array_equal(got, (res + ref).astype(F32))


def _backend(path, dtype, max_context=512):
    _torch()
    from huncho_b200.backend import KevBackend
    return KevBackend(path, device=0, dtype=dtype, max_context=max_context)


def _assert_paired(a, b, tol=1e-4):
    for t in (0.75, 1.0, 2.40605):
        pa, pb = calibration.calibrate(a, t), calibration.calibrate(b, t)
        assert calibration.argmax(pa.tolist()) == calibration.argmax(pb.tolist())
        assert np.abs(pa - pb).max() <= tol, (pa, pb)


@pytest.mark.parametrize("scheme", ["q8_0-fp32", "q4_0-fp32"])
def test_tiny_packed_package_vs_oracle(native_lib, tmp_path, scheme):
    from oracle import kev_oracle as ko
    from huncho_b200.errors import HunchoError
    pkg = quantize.write_package(GOLDEN, scheme, tmp_path / scheme)
    other = "q4_0-fp32" if scheme == "q8_0-fp32" else "q8_0-fp32"
    with pytest.raises(HunchoError):
        _backend(pkg, other)
    b = _backend(pkg, scheme)
    m = ko.load_model(pkg, scheme)
    golden = json.loads((GOLDEN / "golden.json").read_text())
    worst = 0.0
    for case in golden["cases"]:
        for row in case["rows"]:
            tokens, positions = row["tokens"], row["positions"]
            got = b.forward(ForwardInput(tokens, positions)).values[:, 0]
            ref = ko.score_row(m, tokens, positions)
            worst = max(worst, float(np.abs(got - ref).max()))
            _assert_paired(got, ref)
            for out in b.forward_batch([ForwardInput(tokens, positions)] * 2):
                _assert_paired(out.values[:, 0], got)
            boundary = row["prefix_len"]
            parent = b.prefill(tokens[:boundary])
            branch = b.fork(parent)
            suffix = b.forward(ForwardInput(tokens[boundary:], [p - boundary for p in positions],
                                            fork_from=branch)).values[:, 0]
            _assert_paired(suffix, got)
            b.release_cache(branch)
            b.release_cache(parent)
    assert worst < 2e-4, worst


def _ulp_sensitivity(ko, m, rows, positions):
    """How far the oracle's own probabilities move when every packed
    projection's input is changed by one ulp: Q8_0 activation quantization is
    discontinuous, so an input one ulp from a rounding boundary moves its
    block by one quantum."""
    orig = ko.packed_linear

    def nudged(x, pw):
        return orig(np.nextafter(np.asarray(x, F32), F32(np.inf)).astype(F32), pw)

    worst = 0.0
    try:
        for r, p in zip(rows, positions):
            ko.packed_linear = orig
            a = ko.score_row(m, r, p)
            ko.packed_linear = nudged
            b = ko.score_row(m, r, p)
            for t in (0.75, 1.0, 2.40605):
                worst = max(worst, float(np.abs(calibration.calibrate(a, t) - calibration.calibrate(b, t)).max()))
    finally:
        ko.packed_linear = orig
    return worst


def test_synthetic_packed_model_vs_oracle(native_lib, synth_root, tmp_path):
    """A 4-layer model: more activation blocks near a rounding boundary, so the
    gate is the reference's 1e-4 or twice the oracle's own one-ulp sensitivity
    (measured here), whichever is larger; same argmax everywhere."""
    from oracle import kev_oracle as ko
    d = synth.write_model(synth_root / "kev-mini-fp32", name="kev-mini", seed=0, store="fp32")
    pkg = quantize.write_package(d, "q8_0-fp32", tmp_path / "q8")
    b = _backend(pkg, "q8_0-fp32", max_context=2048)
    m = ko.load_model(pkg, "q8_0-fp32")
    wl = synth.make_workload(2, b.vocab_size, seed=6, n_requests=3)
    tol = max(1e-4, 2.0 * _ulp_sensitivity(ko, m, wl.rows, wl.positions))
    got = b.score_packed(*pack_rows(wl.rows, wl.positions))
    k = 0
    for r, p in zip(wl.rows, wl.positions):
        ref = ko.score_row(m, r, p)
        _assert_paired(got[k:k + len(p)], ref, tol)
        k += len(p)
