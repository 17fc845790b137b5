"""Copy the reference's tiny Kev fixture into tests/golden/tiny_kev as a Kev model dir.

The reference fixture (crates/huncho-backend/tests/fixtures/tiny_kev in grafuls/huncho)
is a deterministic 2-layer Qwen3.5 (one DeltaNet and one full-attention layer),
a PEFT LoRA adapter and a pointer head saved by ``torch.save`` as ``head.pt``,
plus ``golden.json`` produced by upstream PyTorch (scripts/generate_kev_fixture.py
in the reference). This script copies the data files unchanged and converts
``head.pt`` into the two files this repository's loaders read:

  pointer_head.safetensors   q.weight, q.bias, k.weight, k.bias (fp32)
  kev_head.json              base, base_revision, head_dim, lora, temperature

The reference reads the same fields from ``head.pt`` (kev.rs:28-165). The
golden file is reduced to the fields the tests use (rows: tokens, positions,
raw logits, probabilities; per-request answers; short_logits).

Usage: python tests/golden/make_tiny_kev.py <reference fixture dir>
"""
import json
import shutil
import sys
from pathlib import Path

import torch
from safetensors.numpy import save_file

if len(sys.argv) != 2:
    sys.exit("usage: python tests/golden/make_tiny_kev.py <reference fixture dir "
             "(crates/huncho-backend/tests/fixtures/tiny_kev of a grafuls/huncho checkout)>")
src = Path(sys.argv[1])
dst = Path(__file__).resolve().parent / "tiny_kev"
dst.mkdir(parents=True, exist_ok=True)
for name in ("config.json", "model.safetensors", "adapter_model.safetensors", "adapter_config.json"):
    shutil.copyfile(src / name, dst / name)

ckpt = torch.load(src / "head.pt", weights_only=True, map_location="cpu")
save_file({k: v.float().contiguous().numpy() for k, v in ckpt["head"].items()},
          str(dst / "pointer_head.safetensors"))
meta = {k: ckpt.get(k) for k in ("base", "base_revision", "head_dim", "lora", "temperature",
                                 "option_isolation", "special_embeddings", "weights_dtype")}
(dst / "kev_head.json").write_text(json.dumps(meta, indent=1) + "\n")

golden = json.loads((src / "golden.json").read_text())
slim = {"generator": {k: golden[k] for k in ("torch", "transformers")},
        "short_logits": golden["short_logits"], "cases": []}
for case in golden["cases"]:
    slim["cases"].append({
        "questions": {k: {"type": q["type"]} for k, q in case["request"]["questions"].items()},
        "rows": [{k: r[k] for k in ("tokens", "positions", "prefix_len", "raw_logits", "probabilities")}
                 for r in case["rows"]],
        "answers": case["answers"],
    })
(dst / "golden.json").write_text(json.dumps(slim) + "\n")
print("wrote", dst)
