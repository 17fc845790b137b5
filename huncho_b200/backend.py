"""KevBackend: huncho-core's `Backend` trait for the Kev scorer, over the C ABI.

Mirrors the trait (crates/huncho-core/src/backend.rs:211-438) as implemented
for Kev by `Qwen3_5Backend` (crates/huncho-backend/src/qwen3_5.rs:2515-3266):
same method names, argument meaning, outputs and error kinds. Every forward
runs on the GPU through libhuncho_kev.so; there is no CPU path.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass, field
from typing import Optional, Sequence

import numpy as np

from . import _native
from .errors import BackendError, PackageError, UnsupportedError

_ERR = {
    _native.HK_ERR_BACKEND: BackendError,
    _native.HK_ERR_UNSUPPORTED: UnsupportedError,
    _native.HK_ERR_PACKAGE: PackageError,
    _native.HK_ERR_CUDA: BackendError,
    _native.HK_ERR_ARGUMENT: BackendError,
}


@dataclass
class ForwardInput:
    """backend.rs:52-75. Positions are relative to `tokens`, sorted ascending."""
    tokens: Sequence[int]
    positions: Sequence[int]
    logit_codes: Optional[Sequence[int]] = None
    qtype: int = 0
    retain_cache: bool = False
    fork_from: Optional[int] = None


@dataclass
class ForwardOutput:
    """ForwardOutput::Logits: one row per readout position, one pointer logit each."""
    positions: list
    values: np.ndarray  # [n_positions, 1] float32


@dataclass
class BatchLimits:
    """backend.rs:108-121."""
    max_rows: int = _native.HK_MAX_ROWS
    max_readouts: Optional[int] = None


@dataclass
class Capabilities:
    id: str
    dtype: str
    max_context: int
    supports_fork: bool
    supports_lora: bool
    families: list
    extra: dict = field(default_factory=dict)


class KevBackend:
    """One Kev scorer on one GPU (a handle of the C ABI)."""

    def __init__(self, model_dir, device: int = 0, dtype: str = "bf16", max_context: int = 8192,
                 _handle=None):
        self._lib = _native.load()
        if dtype not in _native.HK_DTYPE:
            raise UnsupportedError(f"Kev's B200 backend supports fp32, bf16, fp16 or int8w, not `{dtype}`")
        self.model_dir = str(model_dir)
        self.dtype = dtype
        self.device = device
        self._h = ctypes.c_void_p()
        if _handle is not None:
            self._h = _handle
        else:
            rc = self._lib.hk_create(self.model_dir.encode(), device, _native.HK_DTYPE[dtype],
                                     int(max_context), ctypes.byref(self._h))
            if rc != _native.HK_OK:
                raise _ERR.get(rc, BackendError)(self._lib.hk_create_error().decode())
        caps = _native.HkCapabilities()
        self._check(self._lib.hk_capabilities_get(self._h, ctypes.byref(caps)))
        self.max_context = caps.max_context
        self.vocab_size = caps.vocab_size
        self.hidden_size = caps.hidden_size
        self.num_layers = caps.num_layers
        self.pointer_dim = caps.pointer_dim
        self.temperature = float(caps.temperature)
        self.lora_rank = caps.lora_rank

    # ---------------------------------------------------------------- plumbing
    def _check(self, rc: int) -> None:
        if rc != _native.HK_OK:
            raise _ERR.get(rc, BackendError)(self._lib.hk_last_error(self._h).decode())

    def close(self) -> None:
        if self._h:
            self._lib.hk_destroy(self._h)
            self._h = ctypes.c_void_p()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    @property
    def kernel_launches(self) -> int:
        return int(self._lib.hk_kernel_launches(self._h))

    def weight_store(self):
        """(device bytes of the weights, store id); replicas on one GPU share the id."""
        sid = ctypes.c_uint64()
        n = self._lib.hk_weight_bytes(self._h, ctypes.byref(sid))
        return int(n), int(sid.value)

    # ---------------------------------------------------------------- trait
    def id(self) -> str:
        return "b200-kev"

    def capabilities(self) -> Capabilities:
        """qwen3_5.rs:2541-2653 (families [F2], dtype, max_context, device)."""
        return Capabilities(
            id=self.id(), dtype=self.dtype, max_context=self.max_context, supports_fork=True,
            supports_lora=True, families=["F2"],
            extra={"device": f"cuda:{self.device}", "native_execution": "b200-kev-sm100a-v1",
                   "pointer_head_dtype": "fp32", "recurrent_state_dtype": "fp32",
                   **({"weight_quantization": "int8-per-channel-symmetric"} if self.dtype == "int8w" else {})},
        )

    def replica(self, device: Optional[int] = None) -> "KevBackend":
        """The same model (on `device`, default the same GPU) with fresh state.
        On the same GPU the replica shares this handle's weights (one device
        copy); on another GPU the package is loaded there."""
        h = ctypes.c_void_p()
        dev = self.device if device is None else device
        rc = self._lib.hk_replica(self._h, dev, ctypes.byref(h))
        if rc != _native.HK_OK:
            raise _ERR.get(rc, BackendError)(self._lib.hk_create_error().decode())
        r = KevBackend.__new__(KevBackend)
        KevBackend.__init__(r, self.model_dir, dev, self.dtype, self.max_context, _handle=h)
        return r

    def with_kv_page_tokens(self, tokens: int, shuffle_seed: int = 0) -> "KevBackend":
        """Qwen3_5Backend::with_kv_page_tokens (qwen3_5.rs:1773-1809): 0 or a power
        of two in 16..256; a nonzero seed shuffles the pages' block table."""
        self._check(self._lib.hk_set_kv_page_tokens(self._h, int(tokens), int(shuffle_seed)))
        return self

    def supports_batch(self) -> bool:
        return True

    def supports_padded_batch(self) -> bool:
        return True

    def supports_fork(self) -> bool:
        return True

    def supports_fork_batch(self) -> bool:
        return True

    def supports_padded_fork_batch(self) -> bool:
        return True

    def batch_limits(self) -> BatchLimits:
        return BatchLimits()

    def fork_batch_limits(self) -> BatchLimits:
        return BatchLimits()

    def forward(self, inp: ForwardInput) -> ForwardOutput:
        """Backend::forward for one row (qwen3_5.rs:2655-2753). With `fork_from`,
        the tokens continue that branch, positions are relative to them, and
        the branch advances to the continued state once the call succeeds."""
        if inp.retain_cache:
            raise UnsupportedError("use prefill to obtain an explicit cache handle")
        tokens = list(inp.tokens)
        if any(int(t) < 0 or int(t) >= self.vocab_size for t in tokens):
            raise BackendError("Qwen3.5 token ID is outside the vocabulary")
        prefix = self.cache_tokens(inp.fork_from) if inp.fork_from is not None else 0
        positions = [int(p) for p in inp.positions]
        if any(p < 0 or p >= len(tokens) for p in positions):
            raise BackendError("Qwen3.5 readout position is outside the token sequence")
        if prefix + len(tokens) > self.max_context:
            raise BackendError(f"sequence length {prefix + len(tokens)} exceeds max_context {self.max_context}")
        if not positions and inp.fork_from is None:
            return ForwardOutput(positions=[], values=np.zeros((0, 1), np.float32))
        if not tokens:
            raise BackendError("cached continuation requires nonempty suffix tokens")
        if inp.fork_from is None:
            return self._run([tokens], [positions])[0]
        logits, _ = self.score_cached(*pack_rows([tokens], [positions]), parents=[int(inp.fork_from)],
                                      mode=_native.HK_CACHE_CONTINUE)
        return ForwardOutput(positions=positions, values=logits.reshape(-1, 1).copy())

    def forward_batch(self, inputs: Sequence[ForwardInput]) -> list:
        """Equal-length independent rows (qwen3_5.rs:2759-2761 -> 3138-3194)."""
        return self._independent(inputs, padded=False)

    def forward_padded_batch(self, inputs: Sequence[ForwardInput]) -> list:
        """Mixed-length rows; padding is invisible (qwen3_5.rs:2806-2816 -> 3138-3194)."""
        return self._independent(inputs, padded=True)

    # ---------------------------------------------------------------- caches
    def prefill(self, tokens) -> int:
        """Backend::prefill (qwen3_5.rs:2833-2835): a handle for the state after `tokens`."""
        return self.prefill_batch([tokens])[0]

    def prefill_batch(self, rows) -> list:
        """Prefill up to 256 prefixes in one native call; one handle per row."""
        rows = [list(r) for r in rows]
        if not rows or len(rows) > _native.HK_MAX_CACHED_ROWS:
            raise BackendError("cached batches take 1..=256 rows")
        tokens, cu, _, _ = pack_rows(rows, [[] for _ in rows])
        handles = np.zeros(len(rows), np.uint64)
        self._check(self._lib.hk_prefill(
            self._h, len(rows), tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
            cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), handles.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))
        return [int(h) for h in handles]

    def fork(self, handle: int) -> int:
        """Backend::fork (qwen3_5.rs:2818-2831): an isolated branch of the same state."""
        out = ctypes.c_uint64()
        self._check(self._lib.hk_fork(self._h, ctypes.c_uint64(int(handle)), ctypes.byref(out)))
        return int(out.value)

    def release_cache(self, handle: int) -> None:
        """Backend::release_cache (qwen3_5.rs:2837-2846); forks of it stay valid."""
        self._check(self._lib.hk_release_cache(self._h, ctypes.c_uint64(int(handle))))

    def cache_tokens(self, handle: int) -> int:
        tokens, nbytes = ctypes.c_int(), ctypes.c_int64()
        if self._lib.hk_cache_info(self._h, ctypes.c_uint64(int(handle)), ctypes.byref(tokens),
                                   ctypes.byref(nbytes)) != _native.HK_OK:
            raise BackendError("unknown Qwen3.5 cache handle")
        return int(tokens.value)

    def cache_bytes(self, handle: int) -> int:
        tokens, nbytes = ctypes.c_int(), ctypes.c_int64()
        if self._lib.hk_cache_info(self._h, ctypes.c_uint64(int(handle)), ctypes.byref(tokens),
                                   ctypes.byref(nbytes)) != _native.HK_OK:
            raise BackendError("unknown Qwen3.5 cache handle")
        return int(nbytes.value)

    def forward_fork_batch(self, parent: int, inputs: Sequence[ForwardInput], work=None) -> list:
        """Equal-length suffixes of one parent (qwen3_5.rs:2780-2791 -> forward_cached_batch)."""
        return self._fork_batch(parent, inputs, padded=False, work=work)

    def forward_padded_fork_batch(self, parent: int, inputs: Sequence[ForwardInput], work=None) -> list:
        """Mixed-length suffixes of one parent (qwen3_5.rs:2793-2804)."""
        return self._fork_batch(parent, inputs, padded=True, work=work)

    def _fork_batch(self, parent, inputs, padded: bool, work) -> list:
        inputs = list(inputs)
        try:
            prefix = self.cache_tokens(parent)
        except BackendError:
            raise BackendError("unknown Qwen3.5 cache handle") from None
        seq = max((len(i.tokens) for i in inputs), default=0)
        bad = (prefix == 0 or not inputs or len(inputs) > _native.HK_MAX_ROWS or seq == 0
               or prefix + seq > self.max_context)
        for i in inputs:
            if (len(i.tokens) == 0 or (not padded and len(i.tokens) != seq) or i.fork_from is not None
                    or i.retain_cache or i.logit_codes is not None or len(i.positions) == 0
                    or any(int(p) < 0 or int(p) >= len(i.tokens) for p in i.positions)
                    or any(int(t) < 0 or int(t) >= self.vocab_size for t in i.tokens)):
                bad = True
        if bad:
            raise BackendError("Kev branch batches require a complete parent, 1..=64 nonempty valid suffixes "
                               "(equal lengths without padding)")
        rows = [list(i.tokens) for i in inputs]
        pos = [[int(p) for p in i.positions] for i in inputs]
        logits, _ = self.score_cached(*pack_rows(rows, pos), parents=[int(parent)] * len(rows),
                                      mode=_native.HK_CACHE_BRANCH)
        if work is not None:
            work.cache_forks = getattr(work, "cache_forks", 0) + len(rows)
            work.forward_calls = getattr(work, "forward_calls", 0) + 1
        out, k = [], 0
        for p in pos:
            out.append(ForwardOutput(positions=list(p), values=logits[k:k + len(p)].reshape(-1, 1).copy()))
            k += len(p)
        return out

    def score_cached(self, tokens, cu_seqlens, positions, cu_positions, parents=None,
                     mode: int = _native.HK_CACHE_BRANCH):
        """hk_score_cached: rows that may each continue a cached prefix (any
        number of parents per call). Returns (logits, new handles or None)."""
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        cup = np.ascontiguousarray(cu_positions, dtype=np.int32)
        n = len(cu) - 1
        par = None if parents is None else np.ascontiguousarray(parents, dtype=np.uint64)
        handles = np.zeros(max(n, 1), np.uint64)
        out = np.empty(max(int(cup[-1]), 1), np.float32)
        self._check(self._lib.hk_score_cached(
            self._h, n, None if par is None else par.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), int(mode),
            tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)), cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), cup.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_float)), handles.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64))))
        new = [int(h) for h in handles[:n]] if mode == _native.HK_CACHE_PREFILL else None
        return out[:int(cup[-1])], new

    def _independent(self, inputs, padded: bool) -> list:
        inputs = list(inputs)
        if not inputs or len(inputs) > _native.HK_MAX_ROWS:
            raise BackendError("Qwen3.5 batch must contain 1..=64 independent rows")
        seq = max(len(i.tokens) for i in inputs)
        bad = seq == 0 or seq > self.max_context
        for i in inputs:
            if (len(i.tokens) == 0 or (not padded and len(i.tokens) != seq) or i.fork_from is not None
                    or i.retain_cache or any(int(p) < 0 or int(p) >= len(i.tokens) for p in i.positions)
                    or any(int(t) < 0 or int(t) >= self.vocab_size for t in i.tokens)):
                bad = True
        if bad:
            raise BackendError("Qwen3.5 batches require valid independent rows without cache handles; "
                               "ordinary batches require equal lengths")
        return self._run([list(i.tokens) for i in inputs], [[int(p) for p in i.positions] for i in inputs])

    def _run(self, rows, positions) -> list:
        logits = self.score_packed(*pack_rows(rows, positions))
        out, k = [], 0
        for pos in positions:
            out.append(ForwardOutput(positions=list(pos),
                                     values=logits[k:k + len(pos)].reshape(-1, 1).copy()))
            k += len(pos)
        return out

    # ---------------------------------------------------------------- packed API
    def score_packed(self, tokens, cu_seqlens, positions, cu_positions) -> np.ndarray:
        """hk_score: raw pointer logits of every readout position, in input order."""
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        cup = np.ascontiguousarray(cu_positions, dtype=np.int32)
        out = np.empty(max(int(cup[-1]), 1), np.float32)
        self._check(self._lib.hk_score(
            self._h, len(cu) - 1, tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
            cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            cup.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), out.ctypes.data_as(ctypes.POINTER(ctypes.c_float))))
        return out[:int(cup[-1])]

    def score_answers(self, tokens, cu_seqlens, positions, cu_positions, question_types,
                      temperature: Optional[float] = None, with_logits: bool = False):
        """hk_score_answers: one question per row, calibrated on the device.

        Returns (probabilities [sum n_pos] fp32, answers: structured array with
        fields best, status, confidence, value per row[, raw logits]). Question
        types are "choice", "noul" ([no, yes]) or "score", or their HK_QUESTION
        codes; the temperature defaults to the package's.
        """
        tokens = np.ascontiguousarray(tokens, dtype=np.uint32)
        cu = np.ascontiguousarray(cu_seqlens, dtype=np.int32)
        pos = np.ascontiguousarray(positions, dtype=np.int32)
        cup = np.ascontiguousarray(cu_positions, dtype=np.int32)
        qt = np.ascontiguousarray([_native.HK_QUESTION[q] if isinstance(q, str) else int(q)
                                   for q in question_types], dtype=np.int32)
        n_rows = len(cu) - 1
        if len(qt) != n_rows:
            raise BackendError("one question type per row is required")
        t = self.temperature if temperature is None else float(temperature)
        p = int(cup[-1])
        probs = np.empty(max(p, 1), np.float32)
        logits = np.empty(max(p, 1), np.float32) if with_logits else None
        answers = (_native.HkAnswer * max(n_rows, 1))()
        pf = ctypes.POINTER(ctypes.c_float)
        self._check(self._lib.hk_score_answers(
            self._h, n_rows, tokens.ctypes.data_as(ctypes.POINTER(ctypes.c_uint32)),
            cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), pos.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            cup.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), qt.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            ctypes.c_float(t), logits.ctypes.data_as(pf) if with_logits else None, probs.ctypes.data_as(pf),
            answers))
        rec = np.array([(a.best, a.status, a.confidence, a.value) for a in answers[:n_rows]],
                       dtype=[("best", np.int32), ("status", np.int32), ("confidence", np.float32),
                              ("value", np.float32)])
        if with_logits:
            return probs[:p], rec, logits[:p]
        return probs[:p], rec

    def score_device(self, cu_seqlens_host, cu_positions_host, d_tokens: int, d_cu_seqlens: int,
                     d_positions: int, d_out: int, stream: int = 0) -> None:
        """hk_score_device: inputs/outputs are device pointers; asynchronous on `stream`."""
        cu = np.ascontiguousarray(cu_seqlens_host, dtype=np.int32)
        cup = np.ascontiguousarray(cu_positions_host, dtype=np.int32)
        self._check(self._lib.hk_score_device(
            self._h, len(cu) - 1, cu.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)),
            cup.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), ctypes.c_void_p(d_tokens),
            ctypes.c_void_p(d_cu_seqlens), ctypes.c_void_p(d_positions), ctypes.c_void_p(d_out),
            ctypes.c_void_p(stream)))

    PROFILE_CLASSES = ("gemm", "delta", "attention", "delta_prep", "other", "rmsnorm", "attn_prep", "readout",
                       "embed")

    def profile(self, enable: bool) -> None:
        """Bracket every launch with CUDA events (see hk_profile_enable)."""
        self._check(self._lib.hk_profile_enable(self._h, 1 if enable else 0))

    def profile_read(self) -> dict:
        """{class: (milliseconds, algorithmic FLOPs, algorithmic HBM bytes, launches)} since the last read."""
        n = len(self.PROFILE_CLASSES)
        ms, fl, by, cnt = ((ctypes.c_double * n)(), (ctypes.c_double * n)(), (ctypes.c_double * n)(),
                           (ctypes.c_int64 * n)())
        self._check(self._lib.hk_profile_read(self._h, ms, fl, by, cnt, n))
        return {c: (ms[i], fl[i], by[i], cnt[i]) for i, c in enumerate(self.PROFILE_CLASSES)}

    def synchronize(self) -> None:
        self._check(self._lib.hk_synchronize(self._h))


def pack_rows(rows, positions):
    """Pack independent rows into (tokens, cu_seqlens, positions, cu_positions)."""
    cu = np.zeros(len(rows) + 1, np.int32)
    cup = np.zeros(len(rows) + 1, np.int32)
    for i, (r, p) in enumerate(zip(rows, positions)):
        cu[i + 1] = cu[i] + len(r)
        cup[i + 1] = cup[i] + len(p)
    tokens = np.concatenate([np.asarray(r, np.uint32) for r in rows]) if rows else np.zeros(0, np.uint32)
    pos = (np.concatenate([np.asarray(p, np.int32) for p in positions])
           if any(len(p) for p in positions) else np.zeros(0, np.int32))
    return tokens, cu, pos, cup
