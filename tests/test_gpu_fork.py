"""Cached prefixes through the C ABI: prefill, fork, continued branches and
branch batches (hk_score_cached / hk_prefill / hk_fork / hk_release_cache).

The property is the reference's own: a question scored as a continuation of
its request's cached prefix gives the probabilities of the same question
scored as one full row (crates/huncho-backend/tests/prefix_cache.rs:141-205:
prefix lengths 1, 2 and the shared prefix, continuations in chunks of 1, 3
and all at once, probabilities within 1e-4 and the same argmax), and cache
handles are owned and transactional (prefix_cache.rs:208-250).

Half-precision models run the 32-token chunked delta kernel, whose chunk
boundaries move when a row is split into prefix + suffix; their gate is the
bf16 gate against the oracle (2e-3), and the measured gap is far below it.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

from huncho_b200 import _native, calibration, synth
from huncho_b200.backend import ForwardInput, pack_rows

from conftest import GOLDEN


def _backend(path, dtype, max_context=512):
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    from huncho_b200.backend import KevBackend
    return KevBackend(path, device=0, dtype=dtype, max_context=max_context)


def _probs(logits, t):
    return calibration.calibrate(np.asarray(logits, np.float32).reshape(-1), t)


def _assert_close(actual, expected, t, tol):
    pa, pe = _probs(actual, t), _probs(expected, t)
    assert np.abs(pa - pe).max() <= tol, (pa, pe)
    assert calibration.argmax(pa.tolist()) == calibration.argmax(pe.tolist())


@pytest.fixture(scope="module")
def golden():
    import json
    return json.loads((GOLDEN / "golden.json").read_text())


@pytest.mark.parametrize("dtype,tol", [("fp32", 1e-4), ("fp16", 1e-4), ("bf16", 1e-4)])
def test_forks_chunks_and_short_prefixes_match_full_rows(native_lib, golden, dtype, tol):
    b = _backend(GOLDEN, dtype)
    for case in golden["cases"]:
        rows = case["rows"]
        first = rows[0]["tokens"]
        shared = rows[0]["prefix_len"]
        for prefix_len in (1, 2, shared):
            parent = b.prefill(first[:prefix_len])
            assert b.cache_tokens(parent) == prefix_len
            for row in rows:
                tokens, positions = row["tokens"], row["positions"]
                assert tokens[:prefix_len] == first[:prefix_len]
                baseline = b.forward(ForwardInput(tokens, positions)).values
                for chunk in (1, 3, None):
                    branch = b.fork(parent)
                    offset = prefix_len
                    # Chunks before the first readout advance every cache part.
                    while offset < positions[0]:
                        end = positions[0] if chunk is None else min(offset + chunk, positions[0])
                        b.forward(ForwardInput(tokens[offset:end], [], fork_from=branch))
                        offset = end
                    got = b.forward(ForwardInput(tokens[offset:], [p - offset for p in positions],
                                                 fork_from=branch)).values
                    _assert_close(got, baseline, b.temperature, tol)
                    assert b.cache_tokens(branch) == len(tokens)
                    b.release_cache(branch)
            b.release_cache(parent)
            with pytest.raises(Exception):
                b.fork(parent)


def test_cache_handles_are_owned_and_transactional(native_lib):
    from huncho_b200.errors import BackendError
    b = _backend(GOLDEN, "fp32", max_context=16)
    other = _backend(GOLDEN, "fp32", max_context=16)
    with pytest.raises(BackendError):
        b.prefill([])
    with pytest.raises(BackendError):
        b.prefill([1] * 17)
    parent = b.prefill([1, 2])
    branch = b.fork(parent)
    with pytest.raises(BackendError):
        other.fork(parent)
    with pytest.raises(BackendError):
        other.forward(ForwardInput([3], [0], fork_from=branch))
    b.release_cache(parent)
    with pytest.raises(BackendError):
        b.release_cache(parent)
    with pytest.raises(BackendError):  # 2 + 15 > max_context
        b.forward(ForwardInput([1] * 15, [0], fork_from=branch))
    with pytest.raises(BackendError):
        b.forward(ForwardInput([3], [1], fork_from=branch))
    with pytest.raises(BackendError):  # a failed continuation does not advance the branch
        b.forward(ForwardInput([2 ** 31], [0], fork_from=branch))
    with pytest.raises(BackendError):
        b.forward(ForwardInput([], [], fork_from=branch))
    assert b.cache_tokens(branch) == 2
    got = b.forward(ForwardInput([3, 4], [0, 1], fork_from=branch)).values
    base = b.forward(ForwardInput([1, 2, 3, 4], [2, 3])).values
    _assert_close(got, base, b.temperature, 1e-4)
    b.release_cache(branch)
    with pytest.raises(BackendError):
        b.score_cached(*pack_rows([[3]], [[0]]), parents=[branch], mode=_native.HK_CACHE_BRANCH)


def _shared_prefix(rows, positions):
    """Longest common prefix of a request's rows that leaves every readout in the suffix."""
    p = min(len(r) for r in rows)
    for r in rows[1:]:
        p = min(p, next((i for i, (a, c) in enumerate(zip(rows[0], r)) if a != c), p))
    return min([p] + [min(ps) for ps in positions])


def _requests(wl):
    reqs = {}
    for i, r in enumerate(wl.request_of):
        reqs.setdefault(r, []).append(i)
    return [reqs[k] for k in sorted(reqs)]


@pytest.mark.parametrize("name,dtype,store,tol", [("kev-mini", "fp32", "fp32", 1e-4),
                                                  ("kev-mini", "bf16", "bf16", 2e-3),
                                                  ("kev-0.8b-l4", "bf16", "bf16", 2e-3),
                                                  ("kev-0.8b-l4", "int8w", "bf16", 2e-3)])
@pytest.mark.parametrize("page_tokens", [0, 16])
def test_multi_parent_branch_batch_matches_full_rows(native_lib, synth_root, name, dtype, store, tol, page_tokens):
    """The benchmark's request fan-out: every request's shared state prefilled in
    one native call, then every question of every request scored in one call
    as a branch of its own request's prefix."""
    d = synth.write_model(synth_root / f"{name}-{store}", name=name, seed=0, store=store)
    b = _backend(d, dtype, max_context=4096)
    if page_tokens:
        b.with_kv_page_tokens(page_tokens, shuffle_seed=5)
    wl = synth.make_workload(2, b.vocab_size, seed=4, n_requests=6)
    full = b.score_packed(*pack_rows(wl.rows, wl.positions))
    reqs = _requests(wl)
    pre = [_shared_prefix([wl.rows[i] for i in q], [wl.positions[i] for i in q]) for q in reqs]
    handles = b.prefill_batch([wl.rows[q[0]][:p] for q, p in zip(reqs, pre)])
    suffix, spos, parents, order = [], [], [], []
    for q, p, h in zip(reqs, pre, handles):
        for i in q:
            suffix.append(list(wl.rows[i][p:]))
            spos.append([x - p for x in wl.positions[i]])
            parents.append(h)
            order.append(i)
    got, _ = b.score_cached(*pack_rows(suffix, spos), parents=parents, mode=_native.HK_CACHE_BRANCH)
    starts = np.concatenate([[0], np.cumsum([len(p) for p in wl.positions])])
    k, worst = 0, 0.0
    for i, sp in zip(order, spos):
        ref = full[starts[i]:starts[i + 1]]
        mine = got[k:k + len(sp)]
        k += len(sp)
        pa, pe = _probs(mine, b.temperature), _probs(ref, b.temperature)
        worst = max(worst, float(np.abs(pa - pe).max()))
        assert calibration.argmax(pa.tolist()) == calibration.argmax(pe.tolist())
    assert worst <= tol, worst
    for h in handles:  # branches left the parents unchanged
        assert b.cache_tokens(h) == pre[handles.index(h)]
        b.release_cache(h)


def test_fork_batch_apis_match_single_branches(native_lib, synth_root):
    """forward_fork_batch (equal lengths) and forward_padded_fork_batch (mixed)
    equal one-row forwards from forks of the same parent; the parent is left
    unchanged (backend.rs:254-316)."""
    from huncho_b200.errors import BackendError
    d = synth.write_model(synth_root / "kev-0.8b-l4-bf16", name="kev-0.8b-l4", seed=0, store="bf16")
    b = _backend(d, "bf16", max_context=4096)
    rng = np.random.default_rng(2)
    parent = b.prefill(rng.integers(0, b.vocab_size, 150).tolist())
    eq = [ForwardInput(rng.integers(0, b.vocab_size, 12).tolist(), [3, 7, 11]) for _ in range(5)]
    mixed = [ForwardInput(rng.integers(0, b.vocab_size, n).tolist(), [0, n - 1]) for n in (3, 17, 40, 65)]
    for inputs, fn in ((eq, b.forward_fork_batch), (mixed, b.forward_padded_fork_batch)):
        outs = fn(parent, inputs)
        for inp, out in zip(inputs, outs):
            br = b.fork(parent)
            single = b.forward(ForwardInput(inp.tokens, inp.positions, fork_from=br)).values
            b.release_cache(br)
            assert np.abs(single - out.values).max() <= 1e-6
    assert b.cache_tokens(parent) == 150
    with pytest.raises(BackendError):  # unequal lengths without padding
        b.forward_fork_batch(parent, mixed)
    with pytest.raises(BackendError):
        b.forward_fork_batch(parent, [ForwardInput([1, 2], [])])
    b.release_cache(parent)
