"""Seeded synthetic Kev packages and scoring workloads.

There is no network and no released Kev checkpoint here, so the benchmark and
the full-size parity tests run on random-init weights of the named shapes,
written as a regular Kev model directory (config.json, model.safetensors,
pointer_head.safetensors, kev_head.json) that the C ABI and the CPU oracle
both read. Weight init follows the workload definition: N(0, 0.02) for
embeddings, projections and the pointer head; the fixture generator's
nontrivial recurrent and norm parameters (A_log = 0.2, dt_bias = 0.1, norm
weights U(-0.1, 0.1); reference scripts/generate_kev_fixture.py:73-80);
depthwise conv weights U(-0.5, 0.5) (PyTorch's Conv1d bound 1/sqrt(taps)).
"""
from __future__ import annotations

import json
import os
import struct
from dataclasses import dataclass
from pathlib import Path

import numpy as np

SPECS = {
    # Qwen3.5-0.8B-shaped Kev: 24 layers [D, D, D, A] x 6.
    "kev-0.8b": dict(hidden_size=1024, num_hidden_layers=24, num_attention_heads=8, num_key_value_heads=2,
                     head_dim=256, intermediate_size=3584, vocab_size=248320, linear_num_key_heads=16,
                     linear_num_value_heads=16, linear_key_head_dim=128, linear_value_head_dim=128,
                     linear_conv_kernel_dim=4, rope_theta=1.0e7, partial_rotary_factor=0.25,
                     rms_norm_eps=1e-6, full_attention_interval=4, pointer_dim=256, temperature=1.3),
    # Qwen3.5-4B-shaped Kev: 32 layers, 16 q / 4 kv heads, delta 16 k / 32 v heads.
    "kev-4b": dict(hidden_size=2560, num_hidden_layers=32, num_attention_heads=16, num_key_value_heads=4,
                   head_dim=256, intermediate_size=9216, vocab_size=248320, linear_num_key_heads=16,
                   linear_num_value_heads=32, linear_key_head_dim=128, linear_value_head_dim=128,
                   linear_conv_kernel_dim=4, rope_theta=1.0e7, partial_rotary_factor=0.25,
                   rms_norm_eps=1e-6, full_attention_interval=4, pointer_dim=256, temperature=1.3),
    # A 0.8B-layout model with 4 layers and a small vocabulary, for fast full-width parity tests.
    "kev-0.8b-l4": dict(hidden_size=1024, num_hidden_layers=4, num_attention_heads=8, num_key_value_heads=2,
                        head_dim=256, intermediate_size=3584, vocab_size=4096, linear_num_key_heads=16,
                        linear_num_value_heads=16, linear_key_head_dim=128, linear_value_head_dim=128,
                        linear_conv_kernel_dim=4, rope_theta=1.0e7, partial_rotary_factor=0.25,
                        rms_norm_eps=1e-6, full_attention_interval=4, pointer_dim=256, temperature=1.3),
    # Small dims with every structural feature (n_rep 2 in the delta rule, GQA 2:1, partial RoPE).
    "kev-mini": dict(hidden_size=128, num_hidden_layers=4, num_attention_heads=4, num_key_value_heads=2,
                     head_dim=64, intermediate_size=256, vocab_size=512, linear_num_key_heads=2,
                     linear_num_value_heads=4, linear_key_head_dim=32, linear_value_head_dim=32,
                     linear_conv_kernel_dim=4, rope_theta=1.0e7, partial_rotary_factor=0.25,
                     rms_norm_eps=1e-6, full_attention_interval=4, pointer_dim=64, temperature=1.3),
}


def config_json(spec: dict) -> dict:
    """An explicit Qwen3.5 text config (every field the loaders read is pinned)."""
    n = spec["num_hidden_layers"]
    iv = spec["full_attention_interval"]
    return {
        "model_type": "qwen3_5_text",
        "hidden_size": spec["hidden_size"], "num_hidden_layers": n,
        "num_attention_heads": spec["num_attention_heads"], "num_key_value_heads": spec["num_key_value_heads"],
        "head_dim": spec["head_dim"], "intermediate_size": spec["intermediate_size"],
        "vocab_size": spec["vocab_size"], "rms_norm_eps": spec["rms_norm_eps"],
        "layer_types": ["full_attention" if (i + 1) % iv == 0 else "linear_attention" for i in range(n)],
        "linear_conv_kernel_dim": spec["linear_conv_kernel_dim"],
        "linear_key_head_dim": spec["linear_key_head_dim"], "linear_value_head_dim": spec["linear_value_head_dim"],
        "linear_num_key_heads": spec["linear_num_key_heads"],
        "linear_num_value_heads": spec["linear_num_value_heads"],
        "rope_parameters": {"rope_type": "default", "rope_theta": spec["rope_theta"],
                            "partial_rotary_factor": spec["partial_rotary_factor"]},
        "hidden_act": "silu", "attention_bias": False, "tie_word_embeddings": False,
        "max_position_embeddings": 262144,
    }


def _tensor_list(spec: dict):
    """(name, shape, init) for every backbone tensor, in file order."""
    H, F = spec["hidden_size"], spec["intermediate_size"]
    nh, nkv, hd = spec["num_attention_heads"], spec["num_key_value_heads"], spec["head_dim"]
    nk, nv, dk, dv = (spec["linear_num_key_heads"], spec["linear_num_value_heads"],
                      spec["linear_key_head_dim"], spec["linear_value_head_dim"])
    conv = 2 * nk * dk + nv * dv
    taps = spec["linear_conv_kernel_dim"]
    iv = spec["full_attention_interval"]
    P = "model.language_model."
    out = [(P + "embed_tokens.weight", (spec["vocab_size"], H), "normal")]
    for i in range(spec["num_hidden_layers"]):
        p = f"{P}layers.{i}."
        out += [(p + "input_layernorm.weight", (H,), "norm"), (p + "post_attention_layernorm.weight", (H,), "norm")]
        if (i + 1) % iv == 0:
            a = p + "self_attn."
            out += [(a + "q_proj.weight", (nh * hd * 2, H), "normal"), (a + "k_proj.weight", (nkv * hd, H), "normal"),
                    (a + "v_proj.weight", (nkv * hd, H), "normal"), (a + "o_proj.weight", (H, nh * hd), "normal"),
                    (a + "q_norm.weight", (hd,), "norm"), (a + "k_norm.weight", (hd,), "norm")]
        else:
            a = p + "linear_attn."
            out += [(a + "in_proj_qkv.weight", (conv, H), "normal"), (a + "in_proj_z.weight", (nv * dv, H), "normal"),
                    (a + "in_proj_b.weight", (nv, H), "normal"), (a + "in_proj_a.weight", (nv, H), "normal"),
                    (a + "out_proj.weight", (H, nv * dv), "normal"), (a + "conv1d.weight", (conv, 1, taps), "conv"),
                    (a + "A_log", (nv,), "alog"), (a + "dt_bias", (nv,), "dtbias"), (a + "norm.weight", (dv,), "ones")]
        m = p + "mlp."
        out += [(m + "gate_proj.weight", (F, H), "normal"), (m + "up_proj.weight", (F, H), "normal"),
                (m + "down_proj.weight", (H, F), "normal")]
    out.append((P + "norm.weight", (H,), "norm"))
    return out


def _init(rng, shape, kind, conv_bound):
    n = int(np.prod(shape))
    if kind == "normal":
        return (rng.standard_normal(n, dtype=np.float32) * np.float32(0.02)).reshape(shape)
    if kind == "norm":
        return rng.uniform(-0.1, 0.1, n).astype(np.float32).reshape(shape)
    if kind == "conv":
        return rng.uniform(-conv_bound, conv_bound, n).astype(np.float32).reshape(shape)
    if kind == "alog":
        return np.full(shape, 0.2, np.float32)
    if kind == "dtbias":
        return np.full(shape, 0.1, np.float32)
    if kind == "ones":
        return np.ones(shape, np.float32)
    raise ValueError(kind)


def _bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + np.uint32(0x7FFF) + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def _write_safetensors(path: Path, names_shapes, dtype: str, produce) -> None:
    """Stream tensors into a safetensors file; `produce(i)` returns tensor i (fp32)."""
    esz = 2 if dtype == "BF16" else 4
    header, off = {}, 0
    for name, shape in names_shapes:
        nb = int(np.prod(shape)) * esz
        header[name] = {"dtype": dtype, "shape": list(shape), "data_offsets": [off, off + nb]}
        off += nb
    hb = json.dumps(header, separators=(",", ":")).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    tmp = path.with_suffix(".tmp")
    with open(tmp, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for i in range(len(names_shapes)):
            t = produce(i)
            f.write((_bf16_bits(t) if dtype == "BF16" else np.ascontiguousarray(t, np.float32)).tobytes())
    os.replace(tmp, path)


def write_model(out_dir, name: str = "kev-0.8b", seed: int = 0, store: str = "bf16") -> Path:
    """Write a seeded synthetic Kev model directory; reuses a complete one."""
    spec = SPECS[name]
    d = Path(out_dir)
    marker = d / ".complete"
    if marker.exists() and json.loads(marker.read_text()) == {"name": name, "seed": seed, "store": store}:
        return d
    d.mkdir(parents=True, exist_ok=True)
    (d / "config.json").write_text(json.dumps(config_json(spec), indent=1))
    rng = np.random.default_rng(seed)
    tensors = _tensor_list(spec)
    conv_bound = 1.0 / np.sqrt(spec["linear_conv_kernel_dim"])
    st = "BF16" if store == "bf16" else "F32"
    _write_safetensors(d / "model.safetensors", [(n, s) for n, s, _ in tensors], st,
                       lambda i: _init(rng, tensors[i][1], tensors[i][2], conv_bound))
    H, dp = spec["hidden_size"], spec["pointer_dim"]
    head = [("q.weight", (dp, H)), ("q.bias", (dp,)), ("k.weight", (dp, H)), ("k.bias", (dp,))]
    _write_safetensors(d / "pointer_head.safetensors", head, "F32",
                       lambda i: _init(rng, head[i][1], "normal", 0))
    (d / "kev_head.json").write_text(json.dumps({
        "base": f"synthetic/{name}", "base_revision": None, "head_dim": dp, "lora": 1,
        "temperature": spec["temperature"], "option_isolation": False, "special_embeddings": False,
        "weights_dtype": "fp32"}))
    marker.write_text(json.dumps({"name": name, "seed": seed, "store": store}))
    return d


def default_dir(name: str, seed: int, store: str) -> Path:
    root = Path(os.environ.get("HK_SYNTH_DIR", "/tmp/huncho_b200_synth"))
    return root / f"{name}-{store}-seed{seed}"


# ---------------------------------------------------------------- workloads
@dataclass
class Workload:
    """Independent question rows plus the request each row belongs to."""
    name: str
    rows: list        # token lists
    positions: list   # readout positions per row
    qtypes: list      # question type per row
    request_of: list  # request index per row
    n_requests: int

    @property
    def n_tokens(self) -> int:
        return sum(len(r) for r in self.rows)


QUESTION_OPTIONS = {"choice-4": ("choice", 4), "noul": ("noul", 2), "score-5": ("score", 5),
                    "choice-8": ("choice", 8)}


def _row(rng, length: int, n_opt: int, vocab: int):
    """A row of `length` ids; options sit at fixed offsets in the tail (one
    <box_start> opt <box_end> triple each, read at the <box_end>), and the
    decision token is the last one."""
    tail = 3 * n_opt + 2
    if length < tail + 1:
        raise ValueError("row too short for its options")
    toks = rng.integers(0, vocab, size=length, dtype=np.int64).astype(np.uint32)
    base = length - tail
    return toks, [base + 3 * j + 2 for j in range(n_opt)]


def make_workload(cfg: int, vocab: int, seed: int = 0, n_requests: int | None = None) -> Workload:
    """The scoring workloads of the benchmark configurations.

    cfg 1: 1 request x 256 tokens, one 4-option choice.
    cfg 2: 32 requests, lengths U[64, 512]; each asks a 4-option choice, a noul
           and a 5-level score, one row per question over the request's tokens.
    cfg 3: 64 requests x 1024 tokens, one 8-option choice each.
    cfg 4: 8 requests x 8192 tokens, one noul each.
    cfg 5: 4096 requests, lengths log-uniform in [32, 2048], question types
           cycling choice-4 / noul / score-5.
    """
    rng = np.random.default_rng(1000 + seed)
    rows, pos, qt, req = [], [], [], []
    if cfg == 1:
        specs = [(256, ["choice-4"])]
    elif cfg == 2:
        n = n_requests or 32
        specs = [(int(rng.integers(64, 513)), ["choice-4", "noul", "score-5"]) for _ in range(n)]
    elif cfg == 3:
        specs = [(1024, ["choice-8"])] * (n_requests or 64)
    elif cfg == 4:
        specs = [(8192, ["noul"])] * (n_requests or 8)
    elif cfg == 5:
        n = n_requests or 4096
        lens = np.exp(rng.uniform(np.log(32), np.log(2048), n)).astype(int)
        cyc = ["choice-4", "noul", "score-5"]
        specs = [(int(lens[i]), [cyc[i % 3]]) for i in range(n)]
    else:
        raise ValueError(f"unknown workload config {cfg}")
    for r, (length, qs) in enumerate(specs):
        state = rng.integers(0, vocab, size=length, dtype=np.int64).astype(np.uint32)
        for q in qs:
            kind, n_opt = QUESTION_OPTIONS[q]
            toks, p = _row(rng, length, n_opt, vocab)
            toks[: length - (3 * n_opt + 2)] = state[: length - (3 * n_opt + 2)]  # shared request state
            rows.append(toks)
            pos.append(p)
            qt.append(kind)
            req.append(r)
    return Workload(name=f"cfg{cfg}", rows=rows, positions=pos, qtypes=qt, request_of=req, n_requests=len(specs))
