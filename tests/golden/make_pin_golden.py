"""Writes the pin-pipeline fixtures under tests/golden/pin/: a tiny dense model and the
pin the reference's own tool makes of it.

- pin/src/: a two-shard model (index + config.json), seeded.  Tensors cover what
  glint_pin.py:39-44,98-104 decides on: BF16, F16 and F32 linears; kept 1-D norms and
  biases; kept 2-D tensors ("rotary" in the name, or no ".weight" suffix); an I64
  tensor; K = 200 (64-blocks straddle rows); 63 weights (odd: a pad nibble); an
  all-zero linear; and weights drawn N(0, 0.02) with 0.1 % outliers x20, rounded to
  BF16 with RNE.
- pin/single.safetensors: a one-file model (output name model.safetensors).
- pin/ref/, pin/ref_single/: glint_pin.convert(src, out, 64, allow_cpu=True) of the
  reference (Jadon-Fox/glint, imported from its checkout; its host numpy encoder, which
  its tests hold byte-equal to its CUDA encoder), plus dry_run.json, its dry-run plan.
- pin/unpin_bf16/, pin/unpin_single_{bf16,f16,f32}/: the reference's
  glint_unpin.unpin of those pins (dense model back, with the pin's own codebook), and
  unpin.json, its return value.

Run from the repository root in a checkout where the reference's Python is importable:
    python tests/golden/make_pin_golden.py /path/to/reference
"""
from __future__ import annotations

import json
import os
import shutil
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

from glint_b200.st_io import write_file  # noqa: E402


def bf16_bits(x: np.ndarray) -> np.ndarray:
    u = np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)
    return ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype("<u2")


def weights(rng, shape, scale=0.02):
    n = int(np.prod(shape))
    w = rng.normal(0.0, scale, n).astype(np.float32)
    k = max(1, n // 1000)
    w[rng.choice(n, size=k, replace=False)] *= 20.0
    return w.reshape(shape)


def t_bf16(name, w):
    return (name, "BF16", tuple(w.shape), bf16_bits(w).tobytes())


def t_f16(name, w):
    return (name, "F16", tuple(w.shape), w.astype("<f2").tobytes())


def t_f32(name, w):
    return (name, "F32", tuple(w.shape), w.astype("<f4").tobytes())


def make_sources(root: Path) -> None:
    rng = np.random.default_rng(0)
    src = root / "src"
    src.mkdir(parents=True, exist_ok=True)
    shard1 = [
        t_bf16("model.embed_tokens.weight", weights(rng, (48, 64))),
        t_bf16("model.layers.0.input_layernorm.weight", np.ones(64, np.float32) + weights(rng, (64,))),
        t_bf16("model.layers.0.self_attn.q_proj.weight", weights(rng, (64, 64))),
        t_bf16("model.layers.0.self_attn.q_proj.bias", weights(rng, (64,))),
        t_bf16("model.layers.0.self_attn.k_proj.weight", weights(rng, (16, 64))),
        t_f32("model.layers.0.rotary_emb.cos_cached", weights(rng, (8, 16), 1.0)),
        t_bf16("model.layers.0.mlp.down_proj.weight", weights(rng, (64, 200))),
        t_bf16("model.layers.0.self_attn.scales", weights(rng, (4, 64))),
    ]
    shard2 = [
        t_f16("model.layers.1.mlp.up_proj.weight", weights(rng, (40, 64))),
        t_bf16("model.layers.1.odd_proj.weight", weights(rng, (7, 9))),
        t_bf16("model.layers.1.zero_proj.weight", np.zeros((8, 64), np.float32)),
        t_f32("model.norm.weight", np.ones(64, np.float32)),
        ("model.position_ids", "I64", (1, 8), np.arange(8, dtype="<i8").tobytes()),
        t_f32("lm_head.weight", weights(rng, (48, 64))),
    ]
    names = ["model-00001-of-00002.safetensors", "model-00002-of-00002.safetensors"]
    weight_map = {}
    for name, tensors in zip(names, (shard1, shard2)):
        write_file(str(src / name), tensors, {"format": "pt"})
        weight_map.update({t[0]: name for t in tensors})
    (src / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}, indent=2))
    (src / "config.json").write_text(json.dumps({"model_type": "llama", "hidden_size": 64}, indent=2) + "\n")
    write_file(str(root / "single.safetensors"),
               [t_bf16("w.weight", weights(rng, (32, 128))), t_bf16("w.bias", weights(rng, (32,)))])


def run_reference(ref: Path, root: Path) -> None:
    os.environ.pop("GLINT_ENCODE_SO", None)  # the reference's host encoder, not a GPU library
    sys.path.insert(0, str(ref))
    import glint_pin  # noqa: E402  (the reference's tool)
    for src, out in ((root / "src", root / "ref"), (root / "single.safetensors", root / "ref_single")):
        if out.exists():
            shutil.rmtree(out)
        plan = glint_pin.convert(src, out, 64, dry_run=True)
        got = glint_pin.convert(src, out, 64, allow_cpu=True)
        assert got["pin"]["backend"] == "cpu_numpy_f32", got["pin"]["backend"]
        (out / "dry_run.json").write_text(json.dumps(plan, indent=2) + "\n")
        # "src" is the generating machine's absolute path: store a placeholder
        for name in ("pin.json", "CONVERT_REPORT.json"):
            doc = json.loads((out / name).read_text())
            pin = doc["pin"] if "pin" in doc else doc
            pin["src"] = "<src>"
            (out / name).write_text(json.dumps(doc, indent=2) + "\n")


def run_reference_unpin(root: Path) -> None:
    import glint_unpin  # noqa: E402  (the reference's tool; its path was added above)
    for pin_dir, out, dtype in ((root / "ref", root / "unpin_bf16", "BF16"),
                                (root / "ref_single", root / "unpin_single_bf16", "BF16"),
                                (root / "ref_single", root / "unpin_single_f16", "F16"),
                                (root / "ref_single", root / "unpin_single_f32", "F32")):
        if out.exists():
            shutil.rmtree(out)
        got = glint_unpin.unpin(pin_dir, out, dtype)
        got["out"] = "<out>"  # the generating machine's path
        (out / "unpin.json").write_text(json.dumps(got, indent=2) + "\n")


if __name__ == "__main__":
    if len(sys.argv) != 2:
        raise SystemExit(__doc__)
    root = HERE / "pin"
    make_sources(root)
    run_reference(Path(sys.argv[1]), root)
    run_reference_unpin(root)
    print("wrote", root)
