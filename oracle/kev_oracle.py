"""NumPy/C restatement of the reference CPU fp32 Kev forward -- TEST INFRASTRUCTURE ONLY.

Every function cites the reference code it follows (paths relative to the
grafuls/huncho project). Arithmetic is fp32 throughout, as in the reference CPU
fp32 path; the per-token delta-rule recurrence and the causal convolution run
in C (``kev_oracle_kernels.c``) in the reference's exact loop order.

Weights are read from a Kev model directory:
  config.json                      Qwen3.5 text config (qwen3_5.rs:53-171)
  *.safetensors                    base weights; ``adapter_model.safetensors`` and
                                   ``pointer_head.safetensors`` are excluded
                                   (qwen3_5.rs:2440-2446)
  adapter_model.safetensors +
  adapter_config.json              optional PEFT LoRA, merged in fp32 at load
                                   (qwen3_5.rs:1597-1640, 2274-2286)
  pointer_head.safetensors +
  kev_head.json                    the pointer head tensors and metadata of the
                                   reference's ``head.pt`` (kev.rs:28-165)

Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg may use this.
"""
from __future__ import annotations

import ctypes
import json
import math
import os
import struct
import subprocess
from dataclasses import dataclass, field
from pathlib import Path

import numpy as np

F32 = np.float32
_HERE = Path(__file__).resolve().parent
_LIB = None


# ---------------------------------------------------------------------------
# C kernels (reference loop order)
# ---------------------------------------------------------------------------

def build_kernels() -> Path:
    """Compile kev_oracle_kernels.c into oracle/_build (gcc, -ffp-contract=off)."""
    out = _HERE / "_build" / "libkev_oracle.so"
    src = _HERE / "kev_oracle_kernels.c"
    if not out.exists() or out.stat().st_mtime < src.stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return out


def _lib():
    global _LIB
    if _LIB is None:
        path = build_kernels()
        lib = ctypes.CDLL(str(path))
        fp = ctypes.POINTER(ctypes.c_float)
        lib.kev_oracle_delta_recurrent.argtypes = [fp, fp, fp, fp, fp] + [ctypes.c_int] * 4 + [fp, fp]
        lib.kev_oracle_causal_conv.argtypes = [fp, fp, ctypes.c_int, ctypes.c_int, ctypes.c_int, fp]
        lib.kev_oracle_set_threads.argtypes = [ctypes.c_int]
        lib.kev_oracle_set_threads(os.cpu_count() or 1)
        _LIB = lib
    return _LIB


def set_threads(n: int) -> None:
    _lib().kev_oracle_set_threads(int(n))


def _ptr(a: np.ndarray):
    assert a.dtype == F32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


def delta_recurrent(q, k, v, g, beta, state=None):
    """Per-token gated delta rule, qwen3_5.rs:950-987 in the order of delta_cpu.rs:99-136.

    q, k: [heads, T, dk]; v: [heads, T, dv]; g, beta: [heads, T] (fp32).
    Returns (out [heads, T, dv], final state [heads, dk, dv]).
    """
    q, k, v = (np.ascontiguousarray(x, dtype=F32) for x in (q, k, v))
    heads, seq, dk = q.shape
    dv = v.shape[2]
    decay = np.ascontiguousarray(np.exp(g.astype(F32)), dtype=F32)  # delta_cpu.rs:61
    beta = np.ascontiguousarray(beta, dtype=F32)
    st = np.zeros((heads, dk, dv), F32) if state is None else np.array(state, dtype=F32, copy=True)
    out = np.zeros((heads, seq, dv), F32)
    _lib().kev_oracle_delta_recurrent(_ptr(q), _ptr(k), _ptr(v), _ptr(decay), _ptr(beta),
                                      heads, seq, dk, dv, _ptr(st), _ptr(out))
    return out, st


def causal_conv(x, w):
    """Depthwise causal conv, conv_cpu.rs:5-52 (== qwen3_5.rs:817-844 before SiLU).

    x: [channels, T]; w: [channels, taps]. Returns the pre-activation [channels, T].
    """
    x = np.ascontiguousarray(x, dtype=F32)
    w = np.ascontiguousarray(w, dtype=F32)
    c, t = x.shape
    out = np.empty_like(x)
    _lib().kev_oracle_causal_conv(_ptr(x), _ptr(w), c, t, w.shape[1], _ptr(out))
    return out


# ---------------------------------------------------------------------------
# safetensors (read-only; format: 8-byte LE header length, JSON header, data)
# ---------------------------------------------------------------------------

def bf16_round(x: np.ndarray) -> np.ndarray:
    """Round fp32 to the nearest bf16 (ties to even) and return it as fp32."""
    u = np.ascontiguousarray(x, dtype=F32).view(np.uint32)
    lsb = (u >> 16) & 1
    r = ((u + np.uint32(0x7FFF) + lsb) & np.uint32(0xFFFF0000)).astype(np.uint32)
    nan = np.isnan(x)
    if nan.any():
        r = np.where(nan, np.uint32(0x7FC00000), r)
    return r.view(F32)


def read_safetensors(path) -> dict:
    """Return {name: ndarray}; BF16 is widened to fp32 exactly."""
    raw = Path(path).read_bytes()
    (hlen,) = struct.unpack("<Q", raw[:8])
    header = json.loads(raw[8:8 + hlen])
    base = 8 + hlen
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        buf = raw[base + a: base + b]
        shape = tuple(info["shape"])
        dt = info["dtype"]
        if dt == "F32":
            arr = np.frombuffer(buf, dtype="<f4").astype(F32)
        elif dt == "F16":
            arr = np.frombuffer(buf, dtype="<f2").astype(F32)
        elif dt == "BF16":
            arr = (np.frombuffer(buf, dtype="<u2").astype(np.uint32) << 16).view(F32)
        elif dt == "F64":
            arr = np.frombuffer(buf, dtype="<f8").astype(F32)
        elif dt == "I8":
            arr = np.frombuffer(buf, dtype=np.int8).copy()
        else:
            raise ValueError(f"unsupported safetensors dtype {dt} for {name}")
        out[name] = arr.reshape(shape)
    return out


# ---------------------------------------------------------------------------
# Config (qwen3_5.rs:53-171)
# ---------------------------------------------------------------------------

@dataclass
class Config:
    hidden_size: int
    num_hidden_layers: int
    num_attention_heads: int
    num_key_value_heads: int
    head_dim: int
    intermediate_size: int
    vocab_size: int
    rms_norm_eps: float
    layer_types: list
    linear_conv_kernel_dim: int
    linear_key_head_dim: int
    linear_num_key_heads: int
    linear_num_value_heads: int
    linear_value_head_dim: int
    rope_theta: float
    partial_rotary_factor: float

    @staticmethod
    def from_value(v: dict) -> "Config":
        """Config::from_value, qwen3_5.rs:77-164 (defaults included)."""
        t = v.get("text_config", v)
        hidden = int(t.get("hidden_size", 4096))
        nl = int(t.get("num_hidden_layers", 32))
        nh = int(t.get("num_attention_heads", 16))
        lt = t.get("layer_types")
        if lt is not None:
            types = []
            for s in lt:
                if "full_attention" in s:
                    types.append("full")
                elif "linear_attention" in s:
                    types.append("linear")
                else:
                    raise ValueError(f"unknown layer type `{s}`")
        else:
            interval = max(int(t.get("full_attention_interval", 4)), 1)
            types = ["full" if (i + 1) % interval == 0 else "linear" for i in range(nl)]
        rp = t.get("rope_parameters") or {}
        theta = rp.get("rope_theta", t.get("rope_theta", 10000.0))
        prf = rp.get("partial_rotary_factor", t.get("partial_rotary_factor", 1.0))
        return Config(
            hidden_size=hidden, num_hidden_layers=nl, num_attention_heads=nh,
            num_key_value_heads=int(t.get("num_key_value_heads", 4)),
            head_dim=int(t.get("head_dim", hidden // nh)),
            intermediate_size=int(t.get("intermediate_size", 12288)),
            vocab_size=int(t.get("vocab_size", 248320)),
            rms_norm_eps=float(np.float32(t.get("rms_norm_eps", 1e-6))),
            layer_types=types,
            linear_conv_kernel_dim=int(t.get("linear_conv_kernel_dim", 4)),
            linear_key_head_dim=int(t.get("linear_key_head_dim", 128)),
            linear_num_key_heads=int(t.get("linear_num_key_heads", 16)),
            linear_num_value_heads=int(t.get("linear_num_value_heads", 32)),
            linear_value_head_dim=int(t.get("linear_value_head_dim", 128)),
            rope_theta=float(theta), partial_rotary_factor=float(prf),
        )

    def rotary_dim(self) -> int:
        """qwen3_5.rs:167-170: round(head_dim * factor), at least 2, made even."""
        d = int(round(self.head_dim * self.partial_rotary_factor))
        return max(d, 2) & ~1


def canonical_weight_name(name: str):
    """qwen3_5.rs:2496-2512."""
    if name.startswith("model.language_model.") or name.startswith("lm_head."):
        return name
    text = name
    for p in ("language_model.", "model."):
        if name.startswith(p):
            text = name[len(p):]
            break
    if any(text.startswith(p) for p in ("layers.", "embed_tokens.", "norm.")):
        return "model.language_model." + text
    return None


PROJECTIONS = (
    "linear_attn.in_proj_qkv", "linear_attn.in_proj_z", "linear_attn.in_proj_b",
    "linear_attn.in_proj_a", "linear_attn.out_proj", "self_attn.q_proj",
    "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
    "mlp.up_proj", "mlp.down_proj",
)


def is_projection(name: str) -> bool:
    return name.endswith(".weight") and any(f".{p}.weight" in name for p in PROJECTIONS)


def quantize_int8_per_channel(w: np.ndarray):
    """Symmetric per-output-channel int8: scale = max|w| / 127, q = rint(w / scale).

    The scheme BASELINE names for the weight-quantized config (no reference
    counterpart; the reference's own scheme is GGML Q8_0, qwen_quantized.rs).
    All-zero rows get scale 1. Returns (q int8 [out, in], scale fp32 [out]).
    """
    w = w.astype(F32)
    amax = np.max(np.abs(w), axis=1).astype(F32)
    scale = (amax / F32(127.0)).astype(F32)
    scale = np.where(scale == 0, F32(1.0), scale).astype(F32)
    q = np.rint(w / scale[:, None]).astype(F32)
    q = np.clip(q, -127, 127).astype(np.int8)
    return q, scale


@dataclass
class KevModel:
    cfg: Config
    w: dict
    head: dict
    temperature: float
    head_dim: int
    dtype: str
    meta: dict = field(default_factory=dict)


# ---------------------------------------------------------------------------
# Packed (GGML Q8_0 / Q4_0) projections of the reference's quantized profile
# (qwen_quantized.rs; Projection::Packed, qwen3_5.rs:320-369)
# ---------------------------------------------------------------------------

@dataclass
class PackedWeight:
    """One packed projection: int8 block values q [N, nb, 32] (Q4_0 as q - 8),
    fp32 block scales d [N, nb] (the stored fp16 values), logical input width."""
    q: np.ndarray
    d: np.ndarray
    width: int


def q8_0_rows(x):
    """Q8_0 quantization of fp32 rows [M, K] (K % 32 == 0): per block
    d = max|x| / 127, q = roundf(x * (1/d)), d stored as fp16. Returns
    (q int8 [M, nb, 32], d fp32 [M, nb])."""
    x = np.asarray(x, F32)
    m, k = x.shape
    b = x.reshape(m, k // 32, 32)
    amax = np.max(np.abs(b), axis=2).astype(F32)
    d = (amax / F32(127.0)).astype(F32)
    inv = np.zeros_like(d)
    nz = d != 0
    inv[nz] = (F32(1.0) / d[nz]).astype(F32)
    v = (b * inv[:, :, None]).astype(F32).astype(np.float64)
    q = (np.sign(v) * np.floor(np.abs(v) + 0.5)).clip(-128, 127).astype(np.int8)
    return q, d.astype(np.float16).astype(F32)


def packed_linear(x, pw: PackedWeight):
    """candle's CPU QMatMul (the generic vec_dot): the input rows are padded
    with zeros to the packed width and quantized to Q8_0; per output, over the
    blocks in order, sumf += (float(sum_i q_w q_x) * d_w) * d_x in fp32."""
    x = np.asarray(x, F32)
    lead = x.shape[:-1]
    x2 = x.reshape(-1, x.shape[-1])
    nb = pw.q.shape[1]
    if x2.shape[1] != pw.width:
        raise ValueError("packed projection input width mismatch")
    xp = np.zeros((x2.shape[0], nb * 32), F32)
    xp[:, :pw.width] = x2
    qx, dx = q8_0_rows(xp)
    acc = np.zeros((x2.shape[0], pw.q.shape[0]), F32)
    qw = pw.q.astype(np.int32)
    for b in range(nb):
        sumi = qx[:, b, :].astype(np.int32) @ qw[:, b, :].T
        term = ((sumi.astype(F32) * pw.d[None, :, b]).astype(F32) * dx[:, b:b + 1]).astype(F32)
        acc = (acc + term).astype(F32)
    return acc.reshape(*lead, pw.q.shape[0])


def load_packed_model(model_dir, dtype: str) -> KevModel:
    """A packed package (backbone.gguf + pointer head files): dense tensors
    fp32, projections packed; the reference's load_quantized_kev profile
    (fp32 activations, qwen_quantized.rs:395-...)."""
    from huncho_b200 import gguf  # the container format (a file-format contract)
    d = Path(model_dir)
    meta, tensors = gguf.read(d / "backbone.gguf")
    want = {"q8_0-fp32": ("kev-projections-q8_0-fp32-v1", gguf.TYPE_Q8_0),
            "q4_0-fp32": ("kev-projections-q4_0-fp32-v1", gguf.TYPE_Q4_0)}
    if dtype not in want or meta.get("huncho.quantization") != want[dtype][0]:
        raise ValueError(f"artifact profile {meta.get('huncho.quantization')} does not match {dtype}")
    cfg = Config.from_value(json.loads(meta["huncho.config_json"]))
    widths = json.loads(meta["huncho.input_widths"])
    w = {}
    for name, (t, shape, raw) in tensors.items():
        if t == gguf.TYPE_F32:
            w[name] = np.frombuffer(raw, "<f4").astype(F32).reshape(shape)
            continue
        if t != want[dtype][1]:
            raise ValueError(f"{name}: block type {t} in a {dtype} artifact")
        rows, kp = shape
        nb = kp // 32
        per = 34 if t == gguf.TYPE_Q8_0 else 18
        rec = np.frombuffer(raw, np.uint8).reshape(rows, nb, per)
        scale = rec[:, :, :2].copy().view("<f2").reshape(rows, nb).astype(F32)
        if t == gguf.TYPE_Q8_0:
            q = rec[:, :, 2:].copy().view(np.int8)
        else:
            nib = rec[:, :, 2:]
            q = np.concatenate([(nib & 0x0F).astype(np.int16) - 8, (nib >> 4).astype(np.int16) - 8],
                               axis=2).astype(np.int8)
        w[name] = PackedWeight(q=q, d=scale, width=int(widths[name]))
    meta_h = json.loads((d / "kev_head.json").read_text())
    head = {k: v.astype(F32) for k, v in read_safetensors(d / "pointer_head.safetensors").items()}
    return KevModel(cfg=cfg, w=w, head=head, temperature=float(F32(meta_h.get("temperature", 1.0))),
                    head_dim=int(meta_h.get("head_dim", 256)), dtype=dtype, meta=meta_h)


def load_model(model_dir, dtype: str = "fp32") -> KevModel:
    """Load base weights, merge LoRA in fp32, then apply the model dtype.

    Follows load_with_head (qwen3_5.rs:2185-2348): canonical names
    (2496-2512), LoRA merge ``W += (alpha/r) * B @ A`` in fp32 (1597-1640), then
    the cast to the model dtype. ``bf16`` / ``fp16`` round every backbone
    tensor to that type (the reference loader casts all tensors to the model
    dtype); ``int8w`` is
    ``bf16`` with the projection weights instead quantized per output channel
    and dequantized (``q * scale``) for the fp32 math. The pointer head stays
    fp32 (kev.rs:124-165).
    """
    d = Path(model_dir)
    if dtype in ("q8_0-fp32", "q4_0-fp32"):
        return load_packed_model(d, dtype)
    cfg = Config.from_value(json.loads((d / "config.json").read_text()))
    w = {}
    for p in sorted(d.glob("*.safetensors")):
        if p.name in ("adapter_model.safetensors", "pointer_head.safetensors", "joint_head.safetensors"):
            continue
        for name, arr in read_safetensors(p).items():
            k = canonical_weight_name(name)
            if k is None or k.startswith("lm_head."):
                continue
            if k in w:
                raise ValueError(f"duplicate canonical base tensor `{k}`")
            w[k] = arr.astype(F32)
    ad = d / "adapter_model.safetensors"
    if ad.exists():
        acfg = json.loads((d / "adapter_config.json").read_text())
        r = int(acfg.get("r", 0))
        alpha = float(acfg.get("lora_alpha", r))
        scale = F32(alpha / r) if r > 0 else F32(1.0)
        lora = read_safetensors(ad)
        targets = sorted({n[len("base_model.model."):-len(".lora_A.weight")] for n in lora
                          if n.startswith("base_model.model.") and n.endswith(".lora_A.weight")})
        for t in targets:
            a = lora[f"base_model.model.{t}.lora_A.weight"].astype(F32)
            b = lora[f"base_model.model.{t}.lora_B.weight"].astype(F32)
            key = canonical_weight_name(t + ".weight")
            if key is None or key not in w:
                raise ValueError(f"missing base weight for LoRA target `{t}`")
            # delta = (B @ A) * scale; the rank sum runs in ascending order.
            delta = np.zeros((b.shape[0], a.shape[1]), F32)
            for i in range(a.shape[0]):
                delta = (delta + b[:, i:i + 1] * a[i:i + 1, :]).astype(F32)
            w[key] = (w[key] + (delta * scale).astype(F32)).astype(F32)
    if dtype in ("bf16", "int8w"):
        for k in list(w):
            if dtype == "int8w" and is_projection(k):
                q, s = quantize_int8_per_channel(w[k])
                w[k] = (q.astype(F32) * s[:, None]).astype(F32)
            else:
                w[k] = bf16_round(w[k])
    elif dtype == "fp16":
        for k in list(w):
            w[k] = w[k].astype(np.float16).astype(F32)
    elif dtype != "fp32":
        raise ValueError(f"unsupported dtype {dtype}")
    meta = json.loads((d / "kev_head.json").read_text())
    head = {k: v.astype(F32) for k, v in read_safetensors(d / "pointer_head.safetensors").items()}
    return KevModel(cfg=cfg, w=w, head=head, temperature=float(F32(meta.get("temperature", 1.0))),
                    head_dim=int(meta.get("head_dim", 256)), dtype=dtype, meta=meta)


# ---------------------------------------------------------------------------
# Math helpers (qwen3_5.rs:173-283)
# ---------------------------------------------------------------------------

def rms_norm_effective(x, w_eff, eps):
    """qwen3_5.rs:184-190 with w_eff = 1 + w computed in fp32 (qwen3_5.rs:180-182)."""
    x = x.astype(F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    denom = np.sqrt(var + F32(eps)).astype(F32)
    return ((x / denom) * w_eff).astype(F32)


def rms_norm_gated(x, gate, w, eps):
    """qwen3_5.rs:193-201: rms(x) * w * silu(gate); w is not zero-centred."""
    x = x.astype(F32)
    var = np.mean(x * x, axis=-1, keepdims=True, dtype=F32)
    denom = np.sqrt(var + F32(eps)).astype(F32)
    n = ((x / denom) * w).astype(F32)
    return (n * silu(gate.astype(F32))).astype(F32)


def l2norm(x, eps=1e-6):
    """qwen3_5.rs:204-210."""
    x = x.astype(F32)
    inv = (F32(1.0) / np.sqrt(np.sum(x * x, axis=-1, keepdims=True, dtype=F32) + F32(eps))).astype(F32)
    return (x * inv).astype(F32)


def silu(x):
    return (x / (F32(1.0) + np.exp(-x))).astype(F32)


def sigmoid(x):
    return (F32(1.0) / (F32(1.0) + np.exp(-x))).astype(F32)


def softplus(x):
    """qwen3_5.rs:212-214: log(exp(x) + 1)."""
    return np.log(np.exp(x.astype(F32)) + F32(1.0)).astype(F32)


def rotary_cos_sin(cfg: Config, seq: int, offset: int = 0):
    """RotaryEmbedding::new/cos_sin, qwen3_5.rs:225-246 (fp32 tables)."""
    rd = cfg.rotary_dim()
    half = rd // 2
    inv = np.array([np.float32(cfg.rope_theta) ** np.float32(-(2.0 * i) / rd) for i in range(half)], F32)
    t = np.arange(offset, offset + seq, dtype=F32)[:, None]
    freqs = (t * inv[None, :]).astype(F32)
    emb = np.concatenate([freqs, freqs], axis=1)
    return np.cos(emb).astype(F32), np.sin(emb).astype(F32)


def apply_partial_rotary(x, cos, sin, rd):
    """qwen3_5.rs:249-283 for one tensor x [heads, T, hd]."""
    rot = x[..., :rd]
    half = rd // 2
    rh = np.concatenate([-rot[..., half:], rot[..., :half]], axis=-1)
    emb = (rot * cos[None] + rh * sin[None]).astype(F32)
    return np.concatenate([emb, x[..., rd:]], axis=-1).astype(F32)


def linear(x, w):
    if isinstance(w, PackedWeight):
        return packed_linear(x, w)
    return (x.astype(F32) @ w.T.astype(F32)).astype(F32)


# ---------------------------------------------------------------------------
# Layers (qwen3_5.rs:586-1104)
# ---------------------------------------------------------------------------

def linear_attn(m: KevModel, p: str, x, cache=None):
    """LinearAttn::forward, qwen3_5.rs:846-947, for one row x [T, H].

    With `cache` (a dict, the layer's LayerCache): the conv runs over
    [cache["conv"] ; this row's inputs] and keeps the suffix part, the
    recurrence starts from cache["state"], and both are replaced by the state
    after this row (q35:851-866, 929-944)."""
    c, w = m.cfg, m.w
    T = x.shape[0]
    nk, nv = c.linear_num_key_heads, c.linear_num_value_heads
    dk, dv = c.linear_key_head_dim, c.linear_value_head_dim
    key_dim, value_dim = nk * dk, nv * dv
    mixed = linear(x, w[f"{p}.in_proj_qkv.weight"])  # [T, conv_dim]
    cw = w[f"{p}.conv1d.weight"].reshape(mixed.shape[1], -1)
    xt = mixed.T.copy()  # [conv_dim, T]
    hist = cache.get("conv") if cache is not None else None
    hl = 0 if hist is None else hist.shape[1]
    if hl:
        xt = np.ascontiguousarray(np.concatenate([hist, xt], axis=1))
    if cache is not None:
        keep = min(cw.shape[1] - 1, xt.shape[1])
        cache["conv"] = xt[:, xt.shape[1] - keep:].copy()
    conv = causal_conv(xt, cw)[:, hl:]  # [conv_dim, T]
    mixed = silu(conv).T.copy()  # [T, conv_dim]
    q = mixed[:, :key_dim].reshape(T, nk, dk)
    k = mixed[:, key_dim:2 * key_dim].reshape(T, nk, dk)
    v = mixed[:, 2 * key_dim:].reshape(T, nv, dv)
    z = linear(x, w[f"{p}.in_proj_z.weight"]).reshape(T, nv, dv)
    beta = sigmoid(linear(x, w[f"{p}.in_proj_b.weight"]))  # [T, nv]
    a = linear(x, w[f"{p}.in_proj_a.weight"])
    base_g = (-np.exp(w[f"{p}.A_log"].astype(F32))).astype(F32)
    g = (base_g[None, :] * softplus(a + w[f"{p}.dt_bias"][None, :])).astype(F32)
    n_rep = nv // nk if nv % nk == 0 else 1
    if n_rep > 1:
        q = np.repeat(q, n_rep, axis=1)
        k = np.repeat(k, n_rep, axis=1)
    q = q.transpose(1, 0, 2)  # [nv, T, dk]
    k = k.transpose(1, 0, 2)
    v = v.transpose(1, 0, 2)
    scale = F32(1.0 / math.sqrt(dk))
    q = (l2norm(q) * scale).astype(F32)
    k = l2norm(k)
    out, state = delta_recurrent(q, k, v, g.T.copy(), beta.T.copy(),
                                 None if cache is None else cache.get("state"))
    if cache is not None:
        cache["state"] = state
    out = out.transpose(1, 0, 2)  # [T, nv, dv]
    out = rms_norm_gated(out, z, w[f"{p}.norm.weight"], c.rms_norm_eps).reshape(T, value_dim)
    return linear(out, w[f"{p}.out_proj.weight"])


def full_attn(m: KevModel, p: str, x, cos, sin, cache=None):
    """Attention::forward, qwen3_5.rs:586-726 (flat KV, dense causal mask).

    With `cache`: the row continues cache["k"], cache["v"] ([nkv, P, hd], after
    norm and RoPE); cos / sin then cover positions P.., queries see every cached
    key plus their own causal prefix, and the cache grows by this row."""
    c, w = m.cfg, m.w
    T = x.shape[0]
    nh, nkv, hd = c.num_attention_heads, c.num_key_value_heads, c.head_dim
    qg = linear(x, w[f"{p}.q_proj.weight"]).reshape(T, nh, 2 * hd)
    q, gate = qg[..., :hd], qg[..., hd:]
    q = rms_norm_effective(q.transpose(1, 0, 2), F32(1.0) + w[f"{p}.q_norm.weight"], c.rms_norm_eps)
    k = linear(x, w[f"{p}.k_proj.weight"]).reshape(T, nkv, hd).transpose(1, 0, 2)
    k = rms_norm_effective(k, F32(1.0) + w[f"{p}.k_norm.weight"], c.rms_norm_eps)
    v = linear(x, w[f"{p}.v_proj.weight"]).reshape(T, nkv, hd).transpose(1, 0, 2)
    rd = c.rotary_dim()
    q = apply_partial_rotary(q, cos, sin, rd)
    k = apply_partial_rotary(k, cos, sin, rd)
    P = 0
    if cache is not None:
        if "k" in cache:
            P = cache["k"].shape[1]
            k = np.concatenate([cache["k"], k], axis=1)
            v = np.concatenate([cache["v"], v], axis=1)
        cache["k"], cache["v"] = k, v
    n_rep = nh // nkv
    k = np.repeat(k, n_rep, axis=0)
    v = np.repeat(v, n_rep, axis=0)
    scale = F32(1.0 / math.sqrt(hd))
    scores = (np.matmul(q, k.transpose(0, 2, 1)) * scale).astype(F32)
    mask = np.triu(np.full((T, P + T), -np.inf, F32), P + 1)
    scores = scores + mask[None]
    mx = np.max(scores, axis=-1, keepdims=True)
    e = np.exp(scores - mx).astype(F32)
    probs = (e / np.sum(e, axis=-1, keepdims=True, dtype=F32)).astype(F32)
    attn = np.matmul(probs, v).astype(F32).transpose(1, 0, 2)  # [T, nh, hd]
    attn = (attn * sigmoid(gate)).reshape(T, nh * hd)
    return linear(attn, w[f"{p}.o_proj.weight"])


def mlp(m: KevModel, p: str, x):
    """Mlp::forward, qwen3_5.rs:1020-1031."""
    g = silu(linear(x, m.w[f"{p}.gate_proj.weight"]))
    u = linear(x, m.w[f"{p}.up_proj.weight"])
    return linear((g * u).astype(F32), m.w[f"{p}.down_proj.weight"])


def forward_hidden(m: KevModel, ids, cache=None) -> np.ndarray:
    """Model::forward_inner (qwen3_5.rs:1533-1553) for one row: final-normed hidden [T, H].

    `cache` (from new_cache(), or a copy of a prefilled one) continues a cached
    prefix: positions start at cache["tokens"], and the cache advances to the
    state after this row (Model::forward_cached, qwen3_5.rs:1111-1212)."""
    c, w = m.cfg, m.w
    ids = np.asarray(ids, dtype=np.int64)
    if ids.size == 0:
        raise ValueError("empty row")
    if (ids < 0).any() or (ids >= c.vocab_size).any():
        raise ValueError("token id is outside the vocabulary")
    T = ids.shape[0]
    offset = 0 if cache is None else cache["tokens"]
    cos, sin = rotary_cos_sin(c, T, offset)
    x = w["model.language_model.embed_tokens.weight"][ids].astype(F32)
    for i in range(c.num_hidden_layers):
        p = f"model.language_model.layers.{i}"
        lc = None if cache is None else cache["layers"][i]
        h = rms_norm_effective(x, F32(1.0) + w[f"{p}.input_layernorm.weight"], c.rms_norm_eps)
        if c.layer_types[i] == "linear":
            h = linear_attn(m, f"{p}.linear_attn", h, lc)
        else:
            h = full_attn(m, f"{p}.self_attn", h, cos, sin, lc)
        h = (h + x).astype(F32)
        n = rms_norm_effective(h, F32(1.0) + w[f"{p}.post_attention_layernorm.weight"], c.rms_norm_eps)
        x = (mlp(m, f"{p}.mlp", n) + h).astype(F32)
    if cache is not None:
        cache["tokens"] = offset + T
    return rms_norm_effective(x, F32(1.0) + w["model.language_model.norm.weight"], c.rms_norm_eps)


def new_cache(m: KevModel) -> dict:
    """An empty ModelCache (qwen3_5.rs:1120-1125): per-layer dicts, 0 tokens."""
    return {"tokens": 0, "layers": [dict() for _ in range(m.cfg.num_hidden_layers)]}


def copy_cache(cache: dict) -> dict:
    """Fork: an independent branch of the same state (qwen3_5.rs:2818-2831)."""
    return {"tokens": cache["tokens"],
            "layers": [{k: v.copy() for k, v in lc.items()} for lc in cache["layers"]]}


def prefill(m: KevModel, tokens) -> dict:
    """Backend::prefill (qwen3_5.rs:2833-2835): the cache after `tokens`."""
    cache = new_cache(m)
    forward_hidden(m, tokens, cache)
    return cache


def score_branch(m: KevModel, cache: dict, tokens, positions) -> np.ndarray:
    """forward with fork_from on a copy of `cache` (the parent is left as is):
    raw logits of the suffix `tokens` at suffix-relative `positions`."""
    tokens, positions = list(tokens), list(positions)
    if any(p >= len(tokens) or p < 0 for p in positions):
        raise ValueError("readout position is outside the token sequence")
    hidden = forward_hidden(m, tokens, copy_cache(cache))
    return pointer_head(m, hidden[len(tokens) - 1], hidden[positions])


def pointer_head(m: KevModel, decide, options):
    """PointerHead::forward, kev.rs:169-173: (W_k o + b_k) . (W_q d + b_q) / sqrt(d_p), fp32."""
    h = m.head
    q = (decide.astype(F32) @ h["q.weight"].T + h["q.bias"]).astype(F32)
    k = (options.astype(F32) @ h["k.weight"].T + h["k.bias"]).astype(F32)
    scale = F32(1.0 / math.sqrt(m.head_dim))
    return ((k @ q) * scale).astype(F32)


def score_row(m: KevModel, tokens, positions) -> np.ndarray:
    """Qwen3_5Backend::forward + readout (qwen3_5.rs:2655-2753, 3196-3255): raw logits [n_pos]."""
    tokens = list(tokens)
    positions = list(positions)
    if any(p >= len(tokens) or p < 0 for p in positions):
        raise ValueError("readout position is outside the token sequence")
    if not positions:
        return np.zeros((0,), F32)
    hidden = forward_hidden(m, tokens)
    return pointer_head(m, hidden[len(tokens) - 1], hidden[positions])


# ---------------------------------------------------------------------------
# Calibration and answers (huncho-core calibration.rs, engine.rs)
# ---------------------------------------------------------------------------

_libm = ctypes.CDLL("libm.so.6")
_libm.expf.restype = ctypes.c_float
_libm.expf.argtypes = [ctypes.c_float]


def softmax_temperature(logits, temperature) -> np.ndarray:
    """calibration.rs:43-64: fp32 exp of (l - max) * (1/T); fp64 sum and divide; fp32 result.
    The fp32 exp is the C library's expf, which Rust's f32::exp calls on Linux."""
    l = np.asarray(logits, dtype=F32)
    if l.size == 0:
        return l.copy()
    inv_t = F32(1.0) / F32(temperature)
    mx = F32(np.max(l))
    with np.errstate(over="ignore", invalid="ignore"):
        z = ((l - mx) * inv_t).astype(F32)
    e = np.array([_libm.expf(v) for v in z.tolist()], dtype=F32)
    s = 0.0
    for v in e:
        s += float(v)
    return np.array([float(v) / s for v in e], dtype=np.float64).astype(F32)


def calibrate(logits, temperature) -> np.ndarray:
    """calibration.rs:172-176, with the validation of 198-218."""
    t = F32(temperature)
    if not np.isfinite(t) or t <= 0:
        raise ValueError(f"temperature must be positive and finite, got {temperature}")
    l = np.asarray(logits, dtype=F32)
    if not np.all(np.isfinite(l)):
        raise ValueError("logits must be finite")
    p = softmax_temperature(l, t)
    if not np.all(np.isfinite(p)):
        raise ValueError("temperature scaling produced nonfinite probabilities")
    return p
