"""The allocation-free pointer readout, through the C ABI.

hk_op_readout_noalloc serves callers that cannot call cudaMalloc (a host that
gives the library only device memory planned ahead from its own pool, or a
serving loop that cannot afford cudaMalloc's implicit device synchronisation):
it keeps its scratch in a fixed library-owned device array instead of taking
scratch buffers. This file checks it against hk_op_readout (the same readout
with caller-provided scratch) on two calls in a row, within the tolerance the
readout's own parity test uses, and checks that sizes beyond the array are
rejected. It is collected last so a failure here comes after every other test.
"""
import ctypes

import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


def _p(t):
    return ctypes.c_void_p(t.data_ptr())


def _inputs(n_tok, hidden, dp, n_dec, n_opt, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    x = torch.randn(n_tok, hidden, device="cuda", generator=g)
    w = 1.0 + 0.1 * torch.rand(hidden, device="cuda", generator=g)
    wq = torch.randn(dp, hidden, device="cuda", generator=g) * 0.02
    wk = torch.randn(dp, hidden, device="cuda", generator=g) * 0.02
    bq = torch.randn(dp, device="cuda", generator=g) * 0.02
    bk = torch.randn(dp, device="cuda", generator=g) * 0.02
    idx = torch.randint(0, n_tok, (n_dec + n_opt,), device="cuda", generator=g, dtype=torch.int64).int()
    opt_dec = torch.randint(0, n_dec, (n_opt,), device="cuda", generator=g, dtype=torch.int64).int()
    return x, w, wq, bq, wk, bk, idx, opt_dec


@pytest.fixture(scope="module")
def lib(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    native_lib.hk_op_readout.argtypes = (
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float] + [ctypes.c_void_p] * 2
        + [ctypes.c_int] * 2 + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 4)
    native_lib.hk_op_readout_noalloc.argtypes = (
        [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float] + [ctypes.c_void_p] * 2
        + [ctypes.c_int] * 2 + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 2)
    native_lib.hk_op_last_error.restype = ctypes.c_char_p
    return native_lib


def _check_against_allocating(lib, n_tok, hidden, dp, n_dec, n_opt, seed, calls=2):
    x, w, wq, bq, wk, bk, idx, opt_dec = _inputs(n_tok, hidden, dp, n_dec, n_opt, seed=seed)
    hn = torch.empty(n_dec + n_opt, hidden, device="cuda")
    proj = torch.empty(n_dec + n_opt, dp, device="cuda")
    ref = torch.empty(n_opt, device="cuda")
    rc = lib.hk_op_readout(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(opt_dec), n_dec, n_opt, _p(wq), _p(bq), _p(wk),
                           _p(bk), dp, _p(hn), _p(proj), _p(ref), None)
    assert rc == 0, lib.hk_op_last_error()
    for _ in range(calls):
        out = torch.full((n_opt,), float("nan"), device="cuda")
        rc = lib.hk_op_readout_noalloc(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(opt_dec), n_dec, n_opt, _p(wq),
                                       _p(bq), _p(wk), _p(bk), dp, _p(out), None)
        assert rc == 0, lib.hk_op_last_error()
        torch.cuda.synchronize()
        torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)


def test_noalloc_readout_matches_allocating_readout_twice(lib):
    _check_against_allocating(lib, 900, 1024, 256, 64, 300, seed=5)


def test_noalloc_readout_at_its_limits_then_smaller(lib):
    """The largest call the array holds (1024 rows of hidden 3584 and their
    512-wide projections: the whole 16 MiB), then a smaller call with other
    shapes over the larger call's leftover contents."""
    _check_against_allocating(lib, 2000, 3584, 512, 100, 924, seed=7, calls=1)
    _check_against_allocating(lib, 50, 256, 64, 3, 11, seed=8)


def test_noalloc_readout_rejects_sizes_beyond_its_scratch(lib):
    n_tok, hidden, dp, n_dec, n_opt = 64, 256, 64, 8, 1017  # 1025 rows > 1024
    x, w, wq, bq, wk, bk, idx, opt_dec = _inputs(n_tok, hidden, dp, n_dec, n_opt, seed=6)
    out = torch.zeros(n_opt, device="cuda")
    rc = lib.hk_op_readout_noalloc(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(opt_dec), n_dec, n_opt, _p(wq), _p(bq),
                                   _p(wk), _p(bk), dp, _p(out), None)
    assert rc == -5
    assert b"fixed scratch" in lib.hk_op_last_error()
    rc = lib.hk_op_readout_noalloc(_p(x), 4096, _p(w), 1e-6, _p(idx), _p(opt_dec), 8, 8, _p(wq), _p(bq), _p(wk),
                                   _p(bk), dp, _p(out), None)
    assert rc == -5


def test_noalloc_readout_rejects_bad_arguments(lib):
    """Options without a decision row and null pointers are argument errors
    (HK_ERR_ARGUMENT) for both readout entry points, before any launch."""
    x, w, wq, bq, wk, bk, idx, opt_dec = _inputs(16, 128, 32, 2, 4, seed=9)
    out = torch.zeros(4, device="cuda")
    scratch = torch.zeros(6, 128, device="cuda")
    rc = lib.hk_op_readout_noalloc(_p(x), 128, _p(w), 1e-6, _p(idx), _p(opt_dec), 0, 4, _p(wq), _p(bq), _p(wk),
                                   _p(bk), 32, _p(out), None)
    assert rc == -5 and b"decision row" in lib.hk_op_last_error()
    rc = lib.hk_op_readout(_p(x), 128, _p(w), 1e-6, _p(idx), _p(opt_dec), 0, 4, _p(wq), _p(bq), _p(wk), _p(bk), 32,
                           _p(scratch), _p(scratch), _p(out), None)
    assert rc == -5
    rc = lib.hk_op_readout_noalloc(None, 128, _p(w), 1e-6, _p(idx), _p(opt_dec), 2, 4, _p(wq), _p(bq), _p(wk),
                                   _p(bk), 32, _p(out), None)
    assert rc == -5 and b"null" in lib.hk_op_last_error()
    rc = lib.hk_op_readout(_p(x), 128, _p(w), 1e-6, _p(idx), _p(opt_dec), 2, 4, _p(wq), _p(bq), _p(wk), _p(bk), 32,
                           None, _p(scratch), _p(out), None)
    assert rc == -5
