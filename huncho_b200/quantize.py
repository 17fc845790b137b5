"""Kev packed backbones: GGML Q8_0 / Q4_0 block quantization and the
reference's converter (crates/huncho-backend/src/qwen_quantized.rs:91-208).

Block formats (32 values per block, row-major blocks along each weight row;
the published GGML reference quantizers, restated):

* Q8_0: amax = max |x|, d = amax / 127, q = round(x * (1/d)) (half away from
  zero; 0 when d = 0), stored as fp16(d) + 32 int8; value = q * d.
* Q4_0: m = the first x of largest |x| (signed), d = m / -8,
  q = min(15, trunc(x * (1/d) + 8.5)), stored as fp16(d) + 16 bytes (value j
  in the low nibble of byte j, value 16 + j in its high nibble); value =
  (q - 8) * d.

Every step runs in fp32 as in the reference (x * (1/d), + 8.5); the packed
projections of a converted artifact are merged with the LoRA adapter in fp32
first, and rows are padded with zeros to a multiple of 32 inputs
(qwen_quantized.rs:116-160). The reference's CPU matmul quantizes each
projection's fp32 input rows to Q8_0 as well and sums, per block,
(integer dot) * d_w * d_x in fp32.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

from . import gguf

F32 = np.float32

SCHEMES = {"q8_0-fp32": gguf.TYPE_Q8_0, "q4_0-fp32": gguf.TYPE_Q4_0}
PROFILES = {"q8_0-fp32": "kev-projections-q8_0-fp32-v1", "q4_0-fp32": "kev-projections-q4_0-fp32-v1"}


def _round_half_away(v: np.ndarray) -> np.ndarray:
    """roundf of fp32 values, exactly (the arithmetic runs in fp64)."""
    v = v.astype(np.float64)
    return np.sign(v) * np.floor(np.abs(v) + 0.5)


def quantize_q8_0(x: np.ndarray):
    """x [rows, K] fp32 (K % 32 == 0) -> (d fp16 [rows, K/32], q int8 [rows, K/32, 32])."""
    x = np.ascontiguousarray(x, dtype=F32)
    rows, k = x.shape
    if k % gguf.BLOCK:
        raise ValueError("Q8_0 rows must be a multiple of 32 wide")
    b = x.reshape(rows, k // gguf.BLOCK, gguf.BLOCK)
    amax = np.max(np.abs(b), axis=2).astype(F32)
    d = (amax / F32(127.0)).astype(F32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, (F32(1.0) / d).astype(F32), F32(0.0)).astype(F32)
    q = _round_half_away((b * inv[:, :, None]).astype(F32))
    q = np.clip(q, -128, 127).astype(np.int8)
    return d.astype(np.float16), q


def dequantize_q8_0(d, q) -> np.ndarray:
    return (q.astype(F32) * d.astype(F32)[:, :, None]).reshape(q.shape[0], -1).astype(F32)


def quantize_q4_0(x: np.ndarray):
    """x [rows, K] fp32 -> (d fp16 [rows, K/32], nibbles uint8 [rows, K/32, 16])."""
    x = np.ascontiguousarray(x, dtype=F32)
    rows, k = x.shape
    if k % gguf.BLOCK:
        raise ValueError("Q4_0 rows must be a multiple of 32 wide")
    b = x.reshape(rows, k // gguf.BLOCK, gguf.BLOCK)
    idx = np.argmax(np.abs(b), axis=2)  # first maximum
    m = np.take_along_axis(b, idx[:, :, None], axis=2)[:, :, 0].astype(F32)
    d = (m / F32(-8.0)).astype(F32)
    with np.errstate(divide="ignore"):
        inv = np.where(d != 0, (F32(1.0) / d).astype(F32), F32(0.0)).astype(F32)
    v = ((b * inv[:, :, None]).astype(F32) + F32(8.5)).astype(F32)
    qi = np.minimum(np.clip(np.trunc(v), 0, 255), 15).astype(np.uint8)
    nib = (qi[:, :, :16] | (qi[:, :, 16:] << 4)).astype(np.uint8)
    return d.astype(np.float16), nib


def q4_values(nib) -> np.ndarray:
    """Signed values (q - 8) [rows, nb, 32] of Q4_0 nibbles."""
    lo = (nib & 0x0F).astype(np.int8) - 8
    hi = (nib >> 4).astype(np.int8) - 8
    return np.concatenate([lo, hi], axis=2).astype(np.int8)


def dequantize_q4_0(d, nib) -> np.ndarray:
    return (q4_values(nib).astype(F32) * d.astype(F32)[:, :, None]).reshape(nib.shape[0], -1).astype(F32)


def pack(ggml_type: int, d, payload) -> bytes:
    """Blocks as stored in GGUF: per block fp16 d then the payload bytes."""
    rows, nb = d.shape
    n = payload.shape[2]
    rec = np.empty((rows, nb, 2 + n), np.uint8)
    rec[:, :, :2] = d.astype("<f2").view(np.uint8).reshape(rows, nb, 2)
    rec[:, :, 2:] = payload.view(np.uint8)
    return rec.tobytes()


def unpack(ggml_type: int, raw: bytes, rows: int, width: int):
    """(d fp16 [rows, nb], payload int8 [rows, nb, 32] or uint8 nibbles [rows, nb, 16])."""
    nb = width // gguf.BLOCK
    per = gguf.BLOCK_BYTES[ggml_type]
    rec = np.frombuffer(raw, np.uint8).reshape(rows, nb, per)
    d = rec[:, :, :2].copy().view("<f2").reshape(rows, nb).astype(np.float16)
    payload = rec[:, :, 2:].copy()
    if ggml_type == gguf.TYPE_Q8_0:
        payload = payload.view(np.int8)
    return d, payload


# ---------------------------------------------------------------------------
# The converter (qwen_quantized.rs:91-208)
# ---------------------------------------------------------------------------

def _read_safetensors(path) -> dict:
    raw = Path(path).read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    header = json.loads(raw[8:8 + n])
    base = 8 + n
    out = {}
    for name, info in header.items():
        if name == "__metadata__":
            continue
        a, b = info["data_offsets"]
        buf = raw[base + a:base + b]
        dt = info["dtype"]
        if dt == "F32":
            arr = np.frombuffer(buf, "<f4")
        elif dt == "F16":
            arr = np.frombuffer(buf, "<f2").astype(F32)
        elif dt == "BF16":
            arr = (np.frombuffer(buf, "<u2").astype(np.uint32) << 16).view(F32)
        else:
            raise ValueError(f"{name}: unsupported dtype {dt}")
        out[name] = arr.astype(F32).reshape(info["shape"])
    return out


def _canonical(name: str):
    """Base tensor names as the reference keys them (qwen3_5.rs:2496-2512)."""
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


def projection_names(cfg: dict) -> list:
    """The packed projections per layer (qwen_quantized.rs:57-86)."""
    names = []
    types = cfg.get("layer_types") or []
    for i in range(int(cfg["num_hidden_layers"])):
        root = f"model.language_model.layers.{i}"
        names += [f"{root}.mlp.{n}.weight" for n in ("gate_proj", "up_proj", "down_proj")]
        full = i < len(types) and types[i] in ("full", "full_attention")
        if full:
            names += [f"{root}.self_attn.{n}.weight" for n in ("q_proj", "k_proj", "v_proj", "o_proj")]
        else:
            names += [f"{root}.linear_attn.{n}.weight"
                      for n in ("in_proj_qkv", "in_proj_z", "in_proj_b", "in_proj_a", "out_proj")]
    return names


def convert_kev(base_dir, adapter_dir, scheme: str, out_path) -> dict:
    """Write the merged text backbone of a Kev package as one GGUF file with
    its projections packed (qwen_quantized.rs:91-193). Returns the conversion
    statistics (counts and bytes). `adapter_dir` None converts a base package
    whose weights are already final (no LoRA merge; the reference always
    merges an adapter of positive rank)."""
    if scheme not in SCHEMES:
        raise ValueError(f"unknown scheme {scheme}")
    base = Path(base_dir)
    adapter = Path(adapter_dir) if adapter_dir is not None else None
    config_text = (base / "config.json").read_text()
    cfg = json.loads(config_text)
    cfg = cfg.get("text_config", cfg)
    w = {}
    for p in sorted(base.glob("*.safetensors")):
        if p.name in ("adapter_model.safetensors", "pointer_head.safetensors", "joint_head.safetensors"):
            continue
        for name, arr in _read_safetensors(p).items():
            k = _canonical(name)
            if k is None or k.startswith("lm_head."):
                continue
            if k in w:
                raise ValueError(f"duplicate canonical base tensor `{k}`")
            w[k] = arr
    lora, scale = {}, F32(1.0)
    if adapter_dir is not None:
        acfg = json.loads((adapter / "adapter_config.json").read_text())
        r = int(acfg.get("r", 0))
        if r <= 0:
            raise ValueError("quantization requires a positive LoRA rank")
        scale = F32(float(acfg.get("lora_alpha", r)) / r)
        lora = _read_safetensors(adapter / "adapter_model.safetensors")
    targets = sorted({n[len("base_model.model."):-len(".lora_A.weight")] for n in lora
                      if n.startswith("base_model.model.") and n.endswith(".lora_A.weight")})
    for t in targets:  # W += (alpha / r) (B @ A), the rank sum in ascending order, fp32
        a = lora[f"base_model.model.{t}.lora_A.weight"]
        b = lora[f"base_model.model.{t}.lora_B.weight"]
        key = _canonical(t + ".weight")
        if key is None or key not in w:
            raise ValueError(f"missing base weight for LoRA target `{t}`")
        delta = np.zeros((b.shape[0], a.shape[1]), F32)
        for i in range(a.shape[0]):
            delta = (delta + b[:, i:i + 1] * a[i:i + 1, :]).astype(F32)
        w[key] = (w[key] + (delta * scale).astype(F32)).astype(F32)
    for name, t in w.items():
        if not np.all(np.isfinite(t)):
            raise ValueError(f"{name}: source weights must be finite")
    qtype = SCHEMES[scheme]
    tensors, widths = {}, {}
    stats = {"scheme": PROFILES[scheme], "projection_count": 0, "source_projection_bytes": 0,
             "packed_projection_bytes": 0, "dense_backbone_bytes": 0}
    for name in projection_names(cfg):
        t = w.pop(name, None)
        if t is None:
            raise ValueError(f"missing projection {name}")
        rows, width = t.shape
        padded = -(-width // gguf.BLOCK) * gguf.BLOCK
        stats["source_projection_bytes"] += t.size * 4
        if padded != width:
            t = np.concatenate([t, np.zeros((rows, padded - width), F32)], axis=1)
        if qtype == gguf.TYPE_Q8_0:
            raw = pack(qtype, *quantize_q8_0(t))
        else:
            raw = pack(qtype, *quantize_q4_0(t))
        tensors[name] = (qtype, (rows, padded), raw)
        widths[name] = width
        stats["projection_count"] += 1
        stats["packed_projection_bytes"] += len(raw)
    for name in sorted(w):
        stats["dense_backbone_bytes"] += w[name].size * 4
        tensors[name] = (gguf.TYPE_F32, tuple(w[name].shape), np.ascontiguousarray(w[name], "<f4").tobytes())
    meta = {"general.architecture": "huncho-kev-qwen3.5", "huncho.quantization": PROFILES[scheme],
            "huncho.config_json": config_text, "huncho.input_widths": json.dumps(widths, sort_keys=True)}
    gguf.write(out_path, meta, dict(sorted(tensors.items())))
    return stats


def write_package(base_dir, scheme: str, out_dir) -> Path:
    """A packed Kev package directory: backbone.gguf (converted from the base
    package and its adapter) plus the base package's pointer head files."""
    base, out = Path(base_dir), Path(out_dir)
    out.mkdir(parents=True, exist_ok=True)
    has_adapter = (base / "adapter_model.safetensors").exists()
    stats = convert_kev(base, base if has_adapter else None, scheme, out / "backbone.gguf")
    for f in ("pointer_head.safetensors", "kev_head.json"):
        (out / f).write_bytes((base / f).read_bytes())
    (out / "quantization.json").write_text(json.dumps(stats, indent=1))
    return out
