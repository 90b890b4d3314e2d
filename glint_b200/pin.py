"""Dense BF16 / F16 / F32 safetensors model -> GLINT pin, encoded on the GPU.

The reference's pin tool (glint_pin.py:1-207 of Jadon-Fox/glint) reads each
tensor into host memory, encodes it through a synchronous host call, computes the
per-linear rmse on the host with numpy (a full expand of every tensor) and holds a
whole output shard in memory before writing it, so an 8B model is host bound.
This pipeline writes the same files, byte for byte:
- the output shards;
- the index (total_size, weight_map);
- the `_glint_cells` codebook tensor;
- the sidecar files;
- pin.json and CONVERT_REPORT.json, with the same fields.

It runs on the GPU through libglint_encode.so:
- shards are memory-mapped, and the next tensor's pages are prefetched;
- every linear is streamed through glint_encode_*_host_sqerr, which encodes it in
  chunks (host->device copy, encode and device->host copy overlapped) and returns
  the rmse's sum of squared errors from the GPU in the same pass;
- each output shard's header is written first, from the known sizes, and writer
  threads put each tensor at its place in the file while the next linear encodes.

Interface: convert(src, out, blocksize, dry_run, allow_cpu, force_python) and main()
mirror glint_pin.py:78-207 (same names, arguments, return value and files). One
difference: there is no host encoder. Without the library or a usable GPU,
convert() raises RuntimeError (also with allow_cpu=True). The reference's own
`glint_pin.py --allow-cpu` is the host path. `backend` reads "cuda_bf16" for BF16
linears, the reference's label for its CUDA path, and "cuda_f32" for F16 / F32
linears, which the reference encodes on the host and which are encoded on the GPU
here.
"""
from __future__ import annotations

import argparse
import ctypes
import json
import math
import shutil
import sys
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import glint_cuda
from .st_io import Reader, ThreadedWriter, Writer

# Which tensors stay dense and which files travel with the pin: the reference's
# rules (glint_pin.py:23-44), since they decide the pin's contents.
PARENT_KEEP = ("norm", "bias", "rotary", "cos_cached", "sin_cached")
INDEX_NAME = "model.safetensors.index.json"
SIDECAR = ("config.json", "generation_config.json", "tokenizer.json", "tokenizer_config.json",
           "special_tokens_map.json", "tokenizer.model", "vocab.json", "merges.txt", "added_tokens.json",
           "chat_template.jinja")
PIN_NOTE = "hole=parent Gaussian cell, plug=child index. H-TILE inflate GLINT_CELLS[h][p]*absmax"


def _is_keep(name: str) -> bool:
    n = name.lower()
    return any(k in n for k in PARENT_KEEP) or name.endswith(".bias")


def _is_linear(name: str, dtype: str, shape) -> bool:
    return dtype in ("BF16", "F16", "F32") and len(shape) == 2 and name.endswith(".weight") and not _is_keep(name)


def resolve_shards(src: Path) -> List[Path]:
    """The shard files a pin reads, in order.  The reference tool's rules
    (glint_pin.py:45-64), in order of precedence:
    - a path that is not a directory is the one shard;
    - a directory's consolidated `model.safetensors`;
    - else the shards its index's weight map names, each once, in name order (a
      named shard that is absent is an error);
    - else the directory's only `.safetensors` file (none or several is an error)."""
    root = Path(src).expanduser().resolve()
    if not root.is_dir():
        return [root]
    files = {p.name: p for p in root.glob("*.safetensors") if p.is_file()}
    if "model.safetensors" in files:
        return [files["model.safetensors"]]
    index = root / INDEX_NAME
    if index.is_file():
        weight_map: Dict[str, str] = json.loads(index.read_text())["weight_map"]
        chosen = [root / name for name in sorted(frozenset(weight_map.values()))]
        absent = [p.name for p in chosen if not p.is_file()]
        if absent:
            raise FileNotFoundError(f"{INDEX_NAME} names missing shards: {absent}")
        return chosen
    if len(files) == 1:
        return list(files.values())
    raise FileNotFoundError(f"need model.safetensors, {INDEX_NAME}, or exactly one .safetensors in {root}")


def _state(blocksize: int, shape, dtype: str) -> bytes:
    """The `.weight.glint_state` bytes of one linear (glint_pin.py:134-137)."""
    return json.dumps({"quant_type": "glint", "blocksize": blocksize, "shape": list(shape), "src_dtype": dtype},
                      separators=(",", ":")).encode()


def _cells_bytes(lib) -> bytes:
    cells = np.empty(256, dtype="<f4")
    if lib.glint_cells_f32(cells.ctypes.data) != 256:
        raise RuntimeError("glint_cells_f32 failed")
    return cells.tobytes()


def _encode(lib, dtype: str, raw: np.ndarray, n: int, bs: int):
    """One linear on the GPU -> (hole, plug, absmax f32, rmse)."""
    hole = np.empty((n + 1) // 2, dtype=np.uint8)
    plug = np.empty((n + 1) // 2, dtype=np.uint8)
    am = np.empty((n + bs - 1) // bs, dtype="<f4")
    sq = ctypes.c_double(0.0)
    if dtype == "BF16":
        fn, src = lib.glint_encode_bf16_host_sqerr, raw
    elif dtype == "F16":  # widened on the host: exact, as glint_np.dense_to_f32 does
        fn, src = lib.glint_encode_f32_host_sqerr, raw.view("<f2").astype("<f4")
    else:
        fn, src = lib.glint_encode_f32_host_sqerr, raw
    rc = fn(src.ctypes.data if n else None, n, bs, hole.ctypes.data if n else None,
            plug.ctypes.data if n else None, am.ctypes.data if n else None, ctypes.byref(sq))
    if rc != 0:
        raise RuntimeError(f"{fn.__name__} rc={rc}")
    return hole, plug, am, (math.sqrt(sq.value / n) if n else 0.0)


def convert(src: Path, out: Path, blocksize: int = 64, dry_run: bool = False, allow_cpu: bool = False,
            force_python: bool = False) -> dict:
    """As glint_pin.convert (glint_pin.py:78-190); allow_cpu / force_python are accepted
    for the same call signature and select nothing: every linear is encoded on the GPU."""
    if blocksize <= 0:
        raise ValueError("blocksize must be positive")
    shards = resolve_shards(src)
    out = Path(out).expanduser().resolve()
    sharded = len(shards) > 1
    plan_linears: List[str] = []
    plan_keep: List[str] = []
    for wf in shards:
        with Reader(str(wf)) as r:
            for e in r.entries:
                (plan_linears if _is_linear(e.name, e.dtype, e.shape) else plan_keep).append(e.name)
    if dry_run:
        return {"schema": "glint_pin_v1", "n_linears": len(plan_linears), "n_keep": len(plan_keep),
                "blocksize": blocksize, "shards": [s.name for s in shards], "linears": plan_linears,
                "cuda": glint_cuda.load() is not None, "numpy": True}
    lib = glint_cuda.require_gpu("GLINT encode", "the reference's glint_pin.py --allow-cpu")
    out.mkdir(parents=True, exist_ok=True)
    reports = []
    weight_map: Dict[str, str] = {}
    total_size = 0
    cells = _cells_bytes(lib)
    for si, wf in enumerate(shards):
        out_name = wf.name if sharded else "model.safetensors"
        with Reader(str(wf)) as r:
            # the shard's output entries, sizes known before any encode
            layout: List[Tuple[str, str, Tuple[int, ...], int]] = []
            for e in r.entries:
                if not _is_linear(e.name, e.dtype, e.shape):
                    layout.append((e.name, e.dtype, e.shape, e.nbytes))
                    continue
                n = int(np.prod(e.shape, dtype=np.int64))
                stem = e.name[: -len(".weight")]
                pk, nam = (n + 1) // 2, (n + blocksize - 1) // blocksize
                st = _state(blocksize, e.shape, e.dtype)
                layout += [(stem + ".weight", "U8", (pk, 1), pk), (stem + ".weight.glint_plug", "U8", (pk, 1), pk),
                           (stem + ".weight.absmax", "F32", (nam,), 4 * nam),
                           (stem + ".weight.glint_state", "U8", (len(st),), len(st))]
            if si == 0:
                layout.append(("_glint_cells", "F32", (16, 16), len(cells)))
            for name, _dt, _sh, nbytes in layout:
                weight_map[name] = out_name
                total_size += nbytes
            wt = ThreadedWriter(Writer(str(out / out_name), layout, {"format": "pt", "quantization": "glint"}))
            ok = False
            try:
                entries = r.entries
                k = 0  # index of the next output entry in `layout`
                for i, e in enumerate(entries):
                    if i + 1 < len(entries):
                        r.prefetch(entries[i + 1])
                    if not _is_linear(e.name, e.dtype, e.shape):
                        wt.put(k, e.name, r.view(e))
                        k += 1
                        continue
                    n = int(np.prod(e.shape, dtype=np.int64))
                    if e.nbytes != n * (2 if e.dtype in ("BF16", "F16") else 4):
                        raise ValueError(f"{wf.name}: {e.name} has {e.nbytes} bytes for shape {list(e.shape)}")
                    hole, plug, am, err = _encode(lib, e.dtype, r.view(e), n, blocksize)
                    stem = e.name[: -len(".weight")]
                    wt.put(k, stem + ".weight", hole)
                    wt.put(k + 1, stem + ".weight.glint_plug", plug)
                    wt.put(k + 2, stem + ".weight.absmax", am)
                    wt.put(k + 3, stem + ".weight.glint_state", _state(blocksize, e.shape, e.dtype))
                    k += 4
                    reports.append({"src": stem, "rmse": err, "shape": list(e.shape),
                                    "backend": "cuda_bf16" if e.dtype == "BF16" else "cuda_f32", "shard": out_name})
                if si == 0:
                    wt.put(k, "_glint_cells", cells)
                ok = True
            finally:
                wt.finish(abort=not ok)
    if sharded:
        index = {"metadata": {"total_size": total_size, "quantization": "glint"}, "weight_map": weight_map}
        (out / INDEX_NAME).write_text(json.dumps(index, indent=2) + "\n")
    src_dir = shards[0].parent
    copied = []
    for side in SIDECAR:
        p = src_dir / side
        if p.is_file() and p.resolve() != (out / side).resolve():
            shutil.copyfile(p, out / side)
            copied.append(side)
    rated = [m["rmse"] for m in reports if m["rmse"] is not None]
    backends = sorted({m["backend"] for m in reports})
    pin = {
        "schema": "glint_pin_v1",
        "src": str(shards[0] if not sharded else src_dir),
        "dest": "glint",
        "n_converted": len(reports),
        "blocksize": blocksize,
        "rmse_mean": (sum(rated) / len(rated)) if rated else None,
        "rmse_max": max(rated) if rated else None,
        "backend": backends[0] if len(backends) == 1 else ("mixed" if backends else None),
        "backends": backends,
        "shards": [s.name for s in shards] if sharded else ["model.safetensors"],
        "sidecar": copied,
        "note": PIN_NOTE,
    }
    (out / "pin.json").write_text(json.dumps(pin, indent=2) + "\n")
    (out / "CONVERT_REPORT.json").write_text(json.dumps({"pin": pin, "modules": reports}, indent=2) + "\n")
    return {"pin": pin, "modules": reports}


def main(argv: Optional[List[str]] = None) -> int:
    p = argparse.ArgumentParser(description="GLINT: BF16 -> hole+plug pin, encoded on the GPU")
    p.add_argument("--src", required=True, help=".safetensors file, model dir, or sharded model dir")
    p.add_argument("--out", required=True)
    p.add_argument("--blocksize", type=int, default=64)
    p.add_argument("--dry-run", action="store_true")
    p.add_argument("--allow-cpu", action="store_true", help="accepted for glint_pin.py compatibility; no effect")
    p.add_argument("--force-python", action="store_true", help="accepted for glint_pin.py compatibility; no effect")
    args = p.parse_args(argv)
    got = convert(Path(args.src), Path(args.out), args.blocksize, args.dry_run, args.allow_cpu, args.force_python)
    print(json.dumps(got if args.dry_run else got["pin"], indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
