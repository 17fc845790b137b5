"""Per-kernel parity on the GPU, through the kernel-level C entry points.

The tensor-core GEMM is checked against an fp32 PyTorch matmul of the same
fp16 operands; the fp32 GEMM against an fp32 matmul with TF32 disabled; the
delta-rule recurrence against the CPU oracle (bit-exact in its exact mode when
the decay is exactly representable); attention against an fp32 PyTorch
reference of qwen3_5.rs:669-714.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

from oracle import kev_oracle as ko


@pytest.fixture(scope="module")
def lib(native_lib):
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    torch.backends.cuda.matmul.allow_tf32 = False
    return native_lib


def _p(t):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def gemm(lib, dtype, epi, x, w, out, scale=None):
    M, K = x.shape
    N = w.shape[0]
    lib.hk_op_gemm.argtypes = [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_int,
                                                   ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p]
    rc = lib.hk_op_gemm(dtype, epi, M, N, K, _p(x), x.stride(0), _p(w), w.stride(0), _p(scale), _p(out),
                        out.stride(0), None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()


SHAPES = [(1, 256, 64), (7, 32, 16), (130, 300, 1024), (257, 512, 72), (300, 8224, 1024), (1000, 1024, 2048),
          (2048, 7168, 1024), (555, 1024, 3584)]


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_store_bf16(lib, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M * 7 + N)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    out = torch.zeros(M, N, device="cuda", dtype=torch.float16)
    gemm(lib, 1, 0, x, w, out)
    ref = x.float() @ w.float().T
    torch.testing.assert_close(out.float(), ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("M,N,K", SHAPES)
def test_tc_gemm_residual_f32(lib, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + N * 3)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    res = torch.randn(M, N, device="cuda", generator=g)
    out = res.clone()
    gemm(lib, 1, 1, x, w, out)
    ref = res + x.float() @ w.float().T
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def test_tc_gemm_scale_and_f32_store(lib):
    g = torch.Generator(device="cuda").manual_seed(5)
    M, N, K = 300, 520, 256
    x = torch.randn(M, K, device="cuda", generator=g).half()
    wq = torch.randint(-127, 128, (N, K), device="cuda", generator=g).float().half()
    scale = torch.rand(N, device="cuda", generator=g) * 1e-3
    out = torch.zeros(M, N, device="cuda")
    gemm(lib, 1, 3, x, wq, out, scale)
    ref = (x.float() @ wq.float().T) * scale
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)


def test_tc_gemm_swiglu(lib):
    g = torch.Generator(device="cuda").manual_seed(9)
    M, F, K = 333, 512, 1024
    x = torch.randn(M, K, device="cuda", generator=g).half()
    gate = (torch.randn(F, K, device="cuda", generator=g) * 0.05).half()
    up = (torch.randn(F, K, device="cuda", generator=g) * 0.05).half()
    w = torch.cat([torch.cat([gate[b:b + 128], up[b:b + 128]]) for b in range(0, F, 128)])
    out = torch.zeros(M, F, device="cuda", dtype=torch.float16)
    gemm(lib, 1, 2, x, w, out)
    gf, uf = x.float() @ gate.float().T, x.float() @ up.float().T
    ref = gf / (1 + torch.exp(-gf)) * uf
    torch.testing.assert_close(out.float(), ref, rtol=2e-2, atol=2e-2)


def test_tc_gemm_repeatable(lib):
    """Same inputs, same bits (no nondeterministic reduction)."""
    g = torch.Generator(device="cuda").manual_seed(11)
    x = torch.randn(777, 1024, device="cuda", generator=g).half()
    w = torch.randn(2048, 1024, device="cuda", generator=g).half()
    a = torch.zeros(777, 2048, device="cuda")
    b = torch.zeros(777, 2048, device="cuda")
    gemm(lib, 1, 3, x, w, a)
    gemm(lib, 1, 3, x, w, b)
    assert torch.equal(a, b)


@pytest.mark.parametrize("M,N,K", [(1, 5, 3), (70, 130, 16), (256, 1000, 1024)])
def test_simt_gemm_f32(lib, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(M + K)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    out = torch.zeros(M, N, device="cuda")
    gemm(lib, 0, 0, x, w, out)
    torch.testing.assert_close(out, x @ w.T, rtol=1e-5, atol=1e-5)
    res = torch.randn(M, N, device="cuda", generator=g)
    out2 = res.clone()
    gemm(lib, 0, 1, x, w, out2)
    torch.testing.assert_close(out2, res + x @ w.T, rtol=1e-5, atol=1e-5)


def _delta_inputs(rng, lens, nk, nv, dk, dv, zero_g=False):
    n = sum(lens)
    q = ko.l2norm(rng.standard_normal((n, nk, dk), dtype=np.float32)) * np.float32(dk ** -0.5)
    k = ko.l2norm(rng.standard_normal((n, nk, dk), dtype=np.float32))
    v = rng.standard_normal((n, nv, dv), dtype=np.float32)
    g = np.zeros((n, nv), np.float32) if zero_g else -rng.random((n, nv), dtype=np.float32) * np.float32(0.5)
    b = rng.random((n, nv), dtype=np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return q.astype(np.float32), k.astype(np.float32), v, g, b, cu


def _delta_oracle(q, k, v, g, b, cu, nk, nv):
    rep = nv // nk
    out = np.zeros_like(v)
    for r in range(len(cu) - 1):
        s, e = cu[r], cu[r + 1]
        qq = np.repeat(q[s:e], rep, axis=1).transpose(1, 0, 2).copy()
        kk = np.repeat(k[s:e], rep, axis=1).transpose(1, 0, 2).copy()
        o, _ = ko.delta_recurrent(qq, kk, v[s:e].transpose(1, 0, 2).copy(), g[s:e].T.copy(), b[s:e].T.copy())
        out[s:e] = o.transpose(1, 0, 2)
    return out


def _run_delta(lib, q, k, v, g, b, cu, nk, nv, exact):
    t = [torch.from_numpy(a).cuda() for a in (q, k, v, g, b, cu)]
    out = torch.zeros_like(t[2])
    lib.hk_op_delta_recurrent.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int] * 6 + [ctypes.c_void_p] * 2
    rc = lib.hk_op_delta_recurrent(*[_p(x) for x in t], len(cu) - 1, nk, nv, q.shape[2], v.shape[2], exact,
                                   _p(out), None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    return out.cpu().numpy()


@pytest.mark.parametrize("exact,nk", [(1, 16), (0, 16), (0, 8)])
def test_delta_recurrence_vs_oracle(lib, exact, nk):
    """exact=1: the per-token kernel in the reference's operation order;
    exact=0: the chunked tensor-core kernel (chunks of 32, a ragged tail, a
    1-token row, rows spanning many chunks; nk < nv exercises the key-head
    repeat)."""
    rng = np.random.default_rng(1)
    nv, dk, dv = 16, 128, 128
    args = _delta_inputs(rng, [37, 1, 130, 64, 300], nk, nv, dk, dv)
    got = _run_delta(lib, *args, nk, nv, exact)
    ref = _delta_oracle(*args, nk, nv)
    if exact:
        np.testing.assert_allclose(got, ref, rtol=1e-4, atol=1e-5)
    else:
        assert np.isfinite(got).all()
        assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


def test_delta_recurrence_exact_order_bitwise(lib):
    """With decay exp(0) = 1 the exact mode reproduces the reference loop bit for bit."""
    rng = np.random.default_rng(2)
    nk, nv, dk, dv = 2, 4, 32, 32
    args = _delta_inputs(rng, [20, 9], nk, nv, dk, dv, zero_g=True)
    got = _run_delta(lib, *args, nk, nv, 1)
    ref = _delta_oracle(*args, nk, nv)
    assert np.array_equal(got, ref)


def _attn_ref(q, k, v, gate, lens, nh, nkv):
    outs = []
    s = 0
    for L in lens:
        qq = q[s:s + L].transpose(0, 1)
        kk = k[s:s + L].transpose(0, 1).repeat_interleave(nh // nkv, 0)
        vv = v[s:s + L].transpose(0, 1).repeat_interleave(nh // nkv, 0)
        sc = qq @ kk.transpose(1, 2) / qq.shape[-1] ** 0.5
        sc = sc + torch.triu(torch.full((L, L), float("-inf"), device=q.device), 1)
        o = (torch.softmax(sc, -1) @ vv).transpose(0, 1)
        outs.append(o * torch.sigmoid(gate[s:s + L]))
        s += L
    return torch.cat(outs).reshape(sum(lens), -1)


@pytest.mark.parametrize("act,hd", [(0, 4), (0, 64), (1, 64), (1, 256)])
def test_attention_vs_torch(lib, act, hd):
    g = torch.Generator(device="cuda").manual_seed(hd)
    nh, nkv = 8, 2
    lens = [5, 70, 1, 33]
    n = sum(lens)
    dt = torch.float32 if act == 0 else torch.float16
    q = torch.randn(n, nh, hd, device="cuda", generator=g).to(dt)
    k = torch.randn(n, nkv, hd, device="cuda", generator=g).to(dt)
    v = torch.randn(n, nkv, hd, device="cuda", generator=g).to(dt)
    proj = torch.randn(n, nh, 2 * hd, device="cuda", generator=g)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    tok_row = torch.tensor(np.repeat(np.arange(len(lens)), lens), dtype=torch.int32, device="cuda")
    out = torch.zeros(n, nh * hd, device="cuda", dtype=dt)
    lib.hk_op_attention.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 2
                                    + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p])
    rc = lib.hk_op_attention(act, _p(q), _p(k), _p(v), _p(proj), nh * 2 * hd, _p(cu), _p(tok_row), n, len(lens),
                             max(lens), nh, nkv, hd, _p(out), nh * hd, None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    ref = _attn_ref(q.float(), k.float(), v.float(), proj.float()[:, :, hd:], lens, nh, nkv)
    tol = 1e-5 if act == 0 else 5e-3
    torch.testing.assert_close(out.float(), ref, rtol=tol, atol=tol)


@pytest.mark.parametrize("hd", [128, 256])
@pytest.mark.parametrize("qscale", [1.0, 6.0])
def test_attention_long_rows_vs_torch(lib, hd, qscale):
    """fp16 attention on rows that span several 128-query and 64-key tiles
    (1-token rows, exact tile boundaries, a ragged 700-token row), with score
    scales that move each row's max by tens of log2 units across tiles (the
    online softmax's rescale path)."""
    g = torch.Generator(device="cuda").manual_seed(hd + int(qscale))
    nh, nkv = 8, 2
    lens = [300, 1, 128, 700, 64, 129]
    n = sum(lens)
    q = (torch.randn(n, nh, hd, device="cuda", generator=g) * qscale).half()
    k = torch.randn(n, nkv, hd, device="cuda", generator=g).half()
    v = torch.randn(n, nkv, hd, device="cuda", generator=g).half()
    proj = torch.randn(n, nh, 2 * hd, device="cuda", generator=g)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(lens)]), dtype=torch.int32, device="cuda")
    tok_row = torch.tensor(np.repeat(np.arange(len(lens)), lens), dtype=torch.int32, device="cuda")
    out = torch.zeros(n, nh * hd, device="cuda", dtype=torch.half)
    lib.hk_op_attention.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 2
                                    + [ctypes.c_int] * 6 + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p])
    rc = lib.hk_op_attention(1, _p(q), _p(k), _p(v), _p(proj), nh * 2 * hd, _p(cu), _p(tok_row), n, len(lens),
                             max(lens), nh, nkv, hd, _p(out), nh * hd, None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    ref = _attn_ref(q.float(), k.float(), v.float(), proj.float()[:, :, hd:], lens, nh, nkv)
    assert torch.isfinite(out.float()).all()
    torch.testing.assert_close(out.float(), ref, rtol=5e-3, atol=5e-3)


def _readout_inputs(g, n_tok, hidden, dp, n_dec, n_opt):
    x = torch.randn(n_tok, hidden, device="cuda", generator=g)
    w = 1.0 + 0.1 * torch.rand(hidden, device="cuda", generator=g)
    wq = torch.randn(dp, hidden, device="cuda", generator=g) * 0.02
    wk = torch.randn(dp, hidden, device="cuda", generator=g) * 0.02
    bq = torch.randn(dp, device="cuda", generator=g) * 0.02
    bk = torch.randn(dp, device="cuda", generator=g) * 0.02
    idx = torch.randint(0, n_tok, (n_dec + n_opt,), device="cuda", generator=g, dtype=torch.int64).int()
    opt_dec = torch.randint(0, n_dec, (n_opt,), device="cuda", generator=g, dtype=torch.int64).int()
    return x, w, wq, bq, wk, bk, idx, opt_dec


def _readout_ref(x, w, wq, bq, wk, bk, idx, opt_dec, n_dec, eps, dp):
    rows = x[idx.long()]
    hn = rows / torch.sqrt((rows * rows).mean(-1, keepdim=True) + eps) * w
    q = hn[:n_dec] @ wq.T + bq
    k = hn[n_dec:] @ wk.T + bk
    return (k * q[opt_dec.long()]).sum(-1) / dp ** 0.5


def test_readout_vs_torch(lib):
    g = torch.Generator(device="cuda").manual_seed(21)
    n_tok, hidden, dp, n_dec, n_opt = 700, 1024, 256, 40, 150
    x, w, wq, bq, wk, bk, idx, opt_dec = _readout_inputs(g, n_tok, hidden, dp, n_dec, n_opt)
    hn = torch.empty(n_dec + n_opt, hidden, device="cuda")
    proj = torch.empty(n_dec + n_opt, dp, device="cuda")
    logits = torch.empty(n_opt, device="cuda")
    lib.hk_op_readout.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float] + [ctypes.c_void_p] * 2
                                  + [ctypes.c_int] * 2 + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 4)
    rc = lib.hk_op_readout(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(opt_dec), n_dec, n_opt, _p(wq), _p(bq), _p(wk),
                           _p(bk), dp, _p(hn), _p(proj), _p(logits), None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    ref = _readout_ref(x, w, wq, bq, wk, bk, idx, opt_dec, n_dec, 1e-6, dp)
    torch.testing.assert_close(logits, ref, rtol=1e-4, atol=1e-5)


def _run_chunked(lib, kernel, q, k, v, g, b, cu, nk, nv, z=None, norm_w=None, eps=1e-6):
    t = [torch.from_numpy(a).cuda() for a in (q, k, v, g, b, cu)]
    n = q.shape[0]
    lib.hk_op_delta_chunked.argtypes = ([ctypes.c_int] + [ctypes.c_void_p] * 6 + [ctypes.c_int] * 3
                                        + [ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float,
                                           ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p])
    if z is None:
        out, zt, nw, ldz, ldo = torch.zeros_like(t[2]), None, None, 0, 0
    else:
        zt, nw = torch.from_numpy(z).cuda(), torch.from_numpy(norm_w).cuda()
        out = torch.zeros(n, nv * 128, dtype=torch.half, device="cuda")
        ldz = ldo = nv * 128
    rc = lib.hk_op_delta_chunked(kernel, *[_p(x) for x in t], len(cu) - 1, nk, nv,
                                 None if zt is None else _p(zt), ldz, None if nw is None else _p(nw), eps,
                                 _p(out), ldo, None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("kernel", [0, 1])
@pytest.mark.parametrize("nk", [16, 8])
def test_delta_chunked_kernels_vs_oracle(lib, kernel, nk):
    """Both chunked forms (0: mma.sync, 32-token chunks; 1: tcgen05, 64-token
    chunks) against the per-token fp32 recurrence: ragged tails, a 1-token
    row, rows of many chunks, and the key-head repeat (nk < nv)."""
    rng = np.random.default_rng(11)
    nv = 16
    args = _delta_inputs(rng, [37, 1, 130, 64, 300], nk, nv, 128, 128)
    got = _run_chunked(lib, kernel, *args, nk, nv)
    ref = _delta_oracle(*args, nk, nv)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 1e-3 * np.abs(ref).max()


@pytest.mark.parametrize("kernel", [0, 1])
def test_delta_chunked_gated_output_vs_oracle(lib, kernel):
    """The fused gated RMSNorm output rms(o) * w * silu(z) (qwen3_5.rs:193-201)
    of both chunked kernels against the oracle's recurrence + rms_norm_gated,
    in fp16 (the out_proj input)."""
    rng = np.random.default_rng(12)
    nk = nv = 16
    q, k, v, g, b, cu = _delta_inputs(rng, [37, 1, 130, 64, 300], nk, nv, 128, 128)
    n = q.shape[0]
    z = rng.standard_normal((n, nv * 128), dtype=np.float32)
    w = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    got = _run_chunked(lib, kernel, q, k, v, g, b, cu, nk, nv, z=z, norm_w=w)
    o = _delta_oracle(q, k, v, g, b, cu, nk, nv)
    ref = ko.rms_norm_gated(o, z.reshape(n, nv, 128), w, 1e-6).reshape(n, nv * 128)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 3e-3 * np.abs(ref).max()


def test_delta_chunked_long_context_stress(lib):
    """The long-context stress configuration at the delta-rule kernel boundary:
    8192-token rows, log-decay g uniform in [-0.1, 0] (a state that remembers
    hundreds of tokens) and beta uniform in (0, 1), chunked tensor-core kernel
    vs the per-token fp32 recurrence."""
    rng = np.random.default_rng(8)
    nk = nv = 16
    n = 2 * 8192
    q = (ko.l2norm(rng.standard_normal((n, nk, 128), dtype=np.float32)) * np.float32(128 ** -0.5)).astype(np.float32)
    k = ko.l2norm(rng.standard_normal((n, nk, 128), dtype=np.float32)).astype(np.float32)
    v = rng.standard_normal((n, nv, 128), dtype=np.float32)
    g = (-rng.random((n, nv), dtype=np.float32) * np.float32(0.1)).astype(np.float32)
    b = rng.uniform(1e-6, 1.0, (n, nv)).astype(np.float32)
    cu = np.array([0, 8192, n], np.int32)
    got = _run_delta(lib, q, k, v, g, b, cu, nk, nv, 0)
    ref = _delta_oracle(q, k, v, g, b, cu, nk, nv)
    assert np.isfinite(got).all()
    assert np.abs(got - ref).max() <= 2e-3 * np.abs(ref).max()


@pytest.mark.parametrize("epi,M,N,K", [(3, 300, 520, 200), (0, 300, 520, 200), (2, 300, 512, 200), (1, 300, 520, 200),
                                       (3, 13, 8224, 1024), (1, 257, 1024, 3584), (2, 2048, 7168, 1024),
                                       (1, 1000, 1024, 2048)])
def test_tc_gemm_cta_pairs_equal_single_cta(lib, epi, M, N, K):
    """The CTA-pair form (cta_group::2, 256 x 256 tiles; hk_op_gemm dtype 2)
    against the single-CTA kernel (dtype 1, which keeps these shapes on single
    CTAs): the same K-block order, so bit-identical outputs for every epilogue,
    ragged M and N included."""
    g = torch.Generator(device="cuda").manual_seed(M + N + K + epi)
    x = torch.randn(M, K, device="cuda", generator=g).half()
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    cols = N // 2 if epi == 2 else N
    dt = torch.float16 if epi in (0, 2) else torch.float32
    base = torch.randn(M, cols, device="cuda", generator=g).to(dt)
    single, pair = base.clone(), base.clone()
    gemm(lib, 1, epi, x, w, single)
    gemm(lib, 2, epi, x, w, pair)
    assert torch.equal(single, pair)


# ---------------------------------------------------------------------------
# The fused delta layer (delta_pipe_kernel), the half-precision models' path
# ---------------------------------------------------------------------------

def _delta_layer_inputs(rng, lens, nk, nv, stress=False):
    """Projection rows q | k | v | z | b | a for hk_op_delta_layer. With
    `stress`, g = base_g * softplus(a + dt_bias) is uniform in [-0.1, -1e-4]
    and beta = sigmoid(b) uniform in (0, 1): the long-context configuration's
    decay and write strengths, set through the kernel's own gate formulas."""
    n = sum(lens)
    conv_dim = 2 * nk * 128 + nv * 128
    ldp = conv_dim + nv * 128 + 2 * nv
    ldp += (-ldp) % 4
    proj = np.zeros((n, ldp), np.float32)
    proj[:, :conv_dim + nv * 128] = rng.standard_normal((n, conv_dim + nv * 128), dtype=np.float32)
    conv_w = rng.uniform(-0.5, 0.5, (conv_dim, 4)).astype(np.float32)
    dt_bias = np.full(nv, 0.1, np.float32)
    if stress:
        base_g = np.full(nv, -1.0, np.float32)
        u = rng.uniform(1e-4, 0.1, (n, nv))
        beta = rng.uniform(1e-6, 1.0 - 1e-6, (n, nv))
        proj[:, conv_dim + nv * 128 + nv:conv_dim + nv * 128 + 2 * nv] = np.log(np.expm1(u)) - 0.1
        proj[:, conv_dim + nv * 128:conv_dim + nv * 128 + nv] = np.log(beta / (1.0 - beta))
    else:
        base_g = (-np.exp(np.full(nv, 0.2, np.float32))).astype(np.float32)
        proj[:, conv_dim + nv * 128:] = rng.standard_normal((n, ldp - conv_dim - nv * 128), dtype=np.float32)
    norm_w = (1.0 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    cu = np.concatenate([[0], np.cumsum(lens)]).astype(np.int32)
    return proj, ldp, conv_w, base_g, dt_bias, norm_w, cu


def _delta_layer_oracle(proj, conv_w, base_g, dt_bias, norm_w, cu, nk, nv, eps=1e-6):
    """LinearAttn::forward between in_proj and out_proj (qwen3_5.rs:846-938) on
    the oracle's pieces: causal conv (conv_cpu.rs order) + SiLU per row, l2norm,
    gates, the per-token recurrence (delta_cpu.rs order), gated RMSNorm."""
    conv_dim = 2 * nk * 128 + nv * 128
    n = proj.shape[0]
    mixed = np.zeros((n, conv_dim), np.float32)
    for r in range(len(cu) - 1):
        s, e = cu[r], cu[r + 1]
        mixed[s:e] = ko.silu(ko.causal_conv(proj[s:e, :conv_dim].T.copy(), conv_w)).T
    q = mixed[:, :nk * 128].reshape(n, nk, 128)
    k = mixed[:, nk * 128:2 * nk * 128].reshape(n, nk, 128)
    v = mixed[:, 2 * nk * 128:].reshape(n, nv, 128).copy()
    q = (ko.l2norm(q) * np.float32(128 ** -0.5)).astype(np.float32)
    k = ko.l2norm(k)
    z = proj[:, conv_dim:conv_dim + nv * 128].reshape(n, nv, 128)
    b = ko.sigmoid(proj[:, conv_dim + nv * 128:conv_dim + nv * 128 + nv])
    a = proj[:, conv_dim + nv * 128 + nv:conv_dim + nv * 128 + 2 * nv]
    g = (base_g[None, :] * ko.softplus(a + dt_bias[None, :])).astype(np.float32)
    o = _delta_oracle(q, k, v, g, b, cu, nk, nv)
    return ko.rms_norm_gated(o, z, norm_w, eps).reshape(n, nv * 128)


def _run_delta_layer(lib, proj, ldp, conv_w, base_g, dt_bias, norm_w, cu, nk, nv, eps=1e-6):
    t = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (proj, cu, conv_w, base_g, dt_bias, norm_w)]
    n = proj.shape[0]
    out = torch.zeros(n, nv * 128, dtype=torch.half, device="cuda")
    lib.hk_op_delta_layer.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 3
                                      + [ctypes.c_void_p] * 4 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                                                                 ctypes.c_void_p])
    rc = lib.hk_op_delta_layer(_p(t[0]), ldp, _p(t[1]), len(cu) - 1, nk, nv, _p(t[2]), _p(t[3]), _p(t[4]), _p(t[5]),
                               eps, _p(out), nv * 128, None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    return out.float().cpu().numpy()


@pytest.mark.parametrize("nk,nv", [(16, 16), (16, 32)])
def test_delta_layer_kernel_vs_oracle(lib, nk, nv):
    """The model's delta kernel (conv + gates + chunked rule + gated norm in one
    launch) on ragged rows: 1-token rows, a row ending exactly on a chunk
    boundary, rows of many chunks; nv = 2 nk is the 4B model's head repeat."""
    rng = np.random.default_rng(31 + nv)
    args = _delta_layer_inputs(rng, [37, 1, 130, 64, 300, 2, 33], nk, nv)
    proj, ldp, conv_w, base_g, dt_bias, norm_w, cu = args
    got = _run_delta_layer(lib, *args, nk, nv)
    ref = _delta_layer_oracle(proj, conv_w, base_g, dt_bias, norm_w, cu, nk, nv)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    print(f"delta layer nk={nk} nv={nv}: max |err| / max |ref| = {err:.3g}")
    # The output is fp16 (half an ulp = 4.9e-4 relative); measured 2.5e-4.
    assert err <= 1e-3


def test_delta_layer_kernel_long_context_stress(lib):
    """The long-context stress configuration at the model's own delta kernel:
    two 8192-token rows, g uniform in [-0.1, 0) and beta uniform in (0, 1)."""
    rng = np.random.default_rng(88)
    nk = nv = 16
    args = _delta_layer_inputs(rng, [8192, 8192], nk, nv, stress=True)
    proj, ldp, conv_w, base_g, dt_bias, norm_w, cu = args
    got = _run_delta_layer(lib, *args, nk, nv)
    ref = _delta_layer_oracle(proj, conv_w, base_g, dt_bias, norm_w, cu, nk, nv)
    assert np.isfinite(got).all()
    err = np.abs(got - ref).max() / np.abs(ref).max()
    print(f"delta layer 2 x 8192 stress: max |err| / max |ref| = {err:.3g}")
    assert err <= 1e-3  # measured 3.0e-4


def test_delta_layer_rejects_bad_shapes(lib):
    lib.hk_op_delta_layer.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p] + [ctypes.c_int] * 3
                                      + [ctypes.c_void_p] * 4 + [ctypes.c_float, ctypes.c_void_p, ctypes.c_int,
                                                                 ctypes.c_void_p])
    x = torch.zeros(64, device="cuda")
    assert lib.hk_op_delta_layer(_p(x), 8224, _p(x), 1, 16, 24, _p(x), _p(x), _p(x), _p(x), 1e-6, _p(x), 2048,
                                 None) == -5  # nv not a multiple of nk
    assert lib.hk_op_delta_layer(_p(x), 100, _p(x), 1, 16, 16, _p(x), _p(x), _p(x), _p(x), 1e-6, _p(x), 2048,
                                 None) == -5  # row stride too small
    assert lib.hk_op_delta_layer(None, 8224, _p(x), 1, 16, 16, _p(x), _p(x), _p(x), _p(x), 1e-6, _p(x), 2048,
                                 None) == -5


def test_readout_bad_decision_index_gives_nan_without_reading(lib):
    """An option whose decision index lies outside [0, n_dec) gets a NaN logit
    (the kernel checks the index and reads nothing for it); the other options
    are unchanged."""
    g = torch.Generator(device="cuda").manual_seed(22)
    n_tok, hidden, dp, n_dec, n_opt = 50, 256, 64, 4, 12
    x, w, wq, bq, wk, bk, idx, opt_dec = _readout_inputs(g, n_tok, hidden, dp, n_dec, n_opt)
    hn = torch.empty(n_dec + n_opt, hidden, device="cuda")
    proj = torch.empty(n_dec + n_opt, dp, device="cuda")
    lib.hk_op_readout.argtypes = ([ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p, ctypes.c_float] + [ctypes.c_void_p] * 2
                                  + [ctypes.c_int] * 2 + [ctypes.c_void_p] * 4 + [ctypes.c_int] + [ctypes.c_void_p] * 4)
    good = torch.empty(n_opt, device="cuda")
    assert lib.hk_op_readout(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(opt_dec), n_dec, n_opt, _p(wq), _p(bq), _p(wk),
                             _p(bk), dp, _p(hn), _p(proj), _p(good), None) == 0
    bad_dec = opt_dec.clone()
    bad_dec[3] = n_dec
    bad_dec[7] = -1
    got = torch.empty(n_opt, device="cuda")
    assert lib.hk_op_readout(_p(x), hidden, _p(w), 1e-6, _p(idx), _p(bad_dec), n_dec, n_opt, _p(wq), _p(bq), _p(wk),
                             _p(bk), dp, _p(hn), _p(proj), _p(got), None) == 0
    torch.cuda.synchronize()
    assert torch.isnan(got[3]) and torch.isnan(got[7])
    keep = [i for i in range(n_opt) if i not in (3, 7)]
    assert torch.equal(got[keep], good[keep])


# ---------------------------------------------------------------------------
# Split-precision projections (fp16 high part + e5m2 low part, fp8 MMAs)
# ---------------------------------------------------------------------------

def _e5m2(t):
    return t.to(torch.float8_e5m2)


def _e4m3(t):
    return t.to(torch.float8_e4m3fn)


def _pad16(t8, cols):
    """An 8-bit [rows, cols] tensor with rows padded to a multiple of 16 bytes."""
    ld = (cols + 15) // 16 * 16
    out = torch.zeros(t8.shape[0], ld, dtype=torch.uint8, device="cuda")
    out[:, :cols] = t8.view(torch.uint8)
    return out, ld


def gemm_split(lib, epi, x_true, w, out, pairs=0, scale=None, out_lo=None):
    M, K = x_true.shape
    N = w.shape[0]
    xh = x_true.half()
    xl, ldxl = _pad16(_e5m2(x_true - xh.float()), K)
    w8, ldw8 = _pad16(_e4m3(w.float()), K)
    lib.hk_op_gemm_split.argtypes = ([ctypes.c_int] * 4 + [ctypes.c_void_p, ctypes.c_int] * 4
                                     + [ctypes.c_void_p] + [ctypes.c_void_p, ctypes.c_int] * 2
                                     + [ctypes.c_int, ctypes.c_void_p])
    olo, ldol = (None, 0) if out_lo is None else out_lo
    rc = lib.hk_op_gemm_split(epi, M, N, K, _p(xh), xh.stride(0), _p(xl), ldxl, _p(w), w.stride(0), _p(w8), ldw8,
                              _p(scale), _p(out), out.stride(0), _p(olo), ldol, pairs, None)
    assert rc == 0, lib.hk_op_last_error()
    torch.cuda.synchronize()
    ref = xh.float() @ w.float().T + _e5m2(x_true - xh.float()).float() @ _e4m3(w.float()).float().T
    return xh, ref


SPLIT_SHAPES = [(7, 32, 16), (130, 300, 1024), (257, 512, 200), (1000, 1024, 2048), (555, 1024, 3584),
                (700, 8224, 1024)]


@pytest.mark.parametrize("pairs", [0, 1])
@pytest.mark.parametrize("M,N,K", SPLIT_SHAPES)
def test_split_gemm_f32_store_and_accuracy(lib, M, N, K, pairs):
    """x w^T + x_lo w8^T accumulated in one fp32 accumulator (kind::f16 then
    kind::f8f6f4 MMAs), single CTAs and CTA pairs, ragged M / N / K: equal to
    the fp32 sum of both products, and much closer to the fp32 product of the
    unrounded input than the fp16 input alone."""
    if pairs and M < 13:
        pytest.skip("CTA pairs run M >= 13 here, as in the pair-kernel test above")
    g = torch.Generator(device="cuda").manual_seed(M + N + K + pairs)
    x = torch.randn(M, K, device="cuda", generator=g) * 2.0
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.02).half()
    out = torch.zeros(M, N, device="cuda")
    xh, ref = gemm_split(lib, 3, x, w, out, pairs=pairs)
    # The tensor cores sum each MMA's products in their own order and width;
    # over K = 3584 that moves outputs of magnitude ~2 by up to ~3e-5.
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-4)
    exact = x @ w.float().T
    err_split = (out - exact).abs().max().item()
    err_f16 = (xh.float() @ w.float().T - exact).abs().max().item()
    assert err_split < err_f16 / 4, (err_split, err_f16)


@pytest.mark.parametrize("M,N,K", [(300, 1024, 2048), (257, 1024, 3584)])
def test_split_gemm_residual(lib, M, N, K):
    g = torch.Generator(device="cuda").manual_seed(3 * M + N)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = (torch.randn(N, K, device="cuda", generator=g) * 0.05).half()
    res = torch.randn(M, N, device="cuda", generator=g)
    out = res.clone()
    _, ref = gemm_split(lib, 1, x, w, out)
    torch.testing.assert_close(out, res + ref, rtol=1e-4, atol=1e-4)


def test_split_gemm_swiglu_writes_low_part(lib):
    """The SwiGLU epilogue on a split-precision input writes the fp16 output
    and the e5m2 rounding of (output - fp16(output)): together they carry the
    SwiGLU value to ~14 bits."""
    g = torch.Generator(device="cuda").manual_seed(19)
    M, F, K = 333, 512, 1024
    x = torch.randn(M, K, device="cuda", generator=g)
    gate = (torch.randn(F, K, device="cuda", generator=g) * 0.05).half()
    up = (torch.randn(F, K, device="cuda", generator=g) * 0.05).half()
    w = torch.cat([torch.cat([gate[b:b + 128], up[b:b + 128]]) for b in range(0, F, 128)])
    out = torch.zeros(M, F, device="cuda", dtype=torch.float16)
    lo = torch.zeros(M, F, device="cuda", dtype=torch.uint8)
    _, acc = gemm_split(lib, 2, x, w, out, out_lo=(lo, F))
    ga = torch.cat([acc[:, b:b + 128] for b in range(0, 2 * F, 256)], 1)
    ua = torch.cat([acc[:, b + 128:b + 256] for b in range(0, 2 * F, 256)], 1)
    y = ga / (1 + torch.exp(-ga)) * ua
    torch.testing.assert_close(out.float(), y, rtol=2e-3, atol=2e-3)
    two = out.float() + lo.view(torch.float8_e5m2).float()
    assert (two - y).abs().max() < (out.float() - y).abs().max() / 3


@pytest.mark.parametrize("M,N,K", [(1, 5, 8), (70, 130, 16), (256, 1000, 1024), (256, 8224, 1024), (600, 1024, 3584)])
def test_tf32x3_gemm_f32(lib, M, N, K):
    """The fp32 model's projections on the tensor cores (hk_op_gemm dtype 3:
    three kind::tf32 products) against an fp32 matmul, store and residual
    epilogues. The operands carry ~2^-20 relative error; the tensor core's
    accumulator adds up to about half an fp32 ulp of the running sum per K step
    (measured: 5.4e-4 on outputs of 15 at K = 3584), so the bound is
    (2e-5 + K 2^-24) of the output scale; a single tf32 product would be ~1e-3
    relative regardless of K."""
    g = torch.Generator(device="cuda").manual_seed(M + 3 * K)
    x = torch.randn(M, K, device="cuda", generator=g)
    w = torch.randn(N, K, device="cuda", generator=g) * 0.05
    ref = x @ w.T
    tol = 2e-5 + K * 2.0 ** -24
    out = torch.zeros(M, N, device="cuda")
    gemm(lib, 3, 3, x, w, out)
    scale = ref.abs().max().item() + 1e-30
    err = (out - ref).abs().max().item()
    print(f"3xTF32 {M}x{N}x{K}: max err {err:.3g} of scale {scale:.3g}")
    assert err <= tol * scale
    res = torch.randn(M, N, device="cuda", generator=g)
    out2 = res.clone()
    gemm(lib, 3, 1, x, w, out2)
    assert (out2 - (res + ref)).abs().max().item() <= tol * (scale + res.abs().max().item())
