"""GLINT pin -> dense safetensors model (BF16 by default), expanded on the GPU.

The reverse of glint_b200.pin, with the interface of the reference's unpin tool
(glint_unpin.py:1-95 of Jadon-Fox/glint, reading pins as glint_pinfile.py:1-76 does):
unpin(pin_dir, out, dtype) and main() take the same arguments and return the same
dict. They write the same files, byte for byte:
- every linear expanded to `dtype` under its original name and shape;
- every other tensor copied through;
- `_glint_cells` and the plug / absmax / state tensors dropped;
- one output shard per pin shard, metadata {"format": "pt", "unpinned_from": "glint"};
- an index when there are several shards, and the pin's sidecar files.

Where the reference expands each module with numpy on the host, here the planes
stream from the memory-mapped pin through the library's chunked host pipeline
(glint_expand_packed_to_bf16_host / _f32_host: copies in, the expand kernel and
copies out overlapped). Each output shard's header is written first, and writer
threads place each tensor at its offset while the next one expands. BF16 is the
kernel's own rounding, the reference's f32_to_bf16_bytes rule (RNE; NaN ->
(bits >> 16) | 0x40). F16 rounds the GPU's f32 values on the host with numpy, as the
reference does.

The kernels carry the compiled codebook. A pin whose `_glint_cells` differs from it
is refused with RuntimeError (the reference's tool, which reads the pin's table, is
the path for such pins), as is a machine without a usable GPU.
"""
from __future__ import annotations

import argparse
import json
import shutil
import sys
from pathlib import Path
from typing import Dict, List, Optional, Tuple

import numpy as np

from . import glint_cuda
from .pin import INDEX_NAME
from .st_io import Entry, Reader, ThreadedWriter, Writer

DTYPES = ("BF16", "F16", "F32")
STATE_SUFFIX = ".weight.glint_state"
_WIDTH = {"BF16": 2, "F16": 2, "F32": 4}


def _module_names(stem: str) -> Tuple[str, str, str, str]:
    w = stem + ".weight"
    return w, w + ".glint_plug", w + ".absmax", stem + STATE_SUFFIX


def _expand(lib, state: dict, hole: np.ndarray, plug: np.ndarray, am: np.ndarray, dtype: str) -> np.ndarray:
    """One module on the GPU -> its dense bytes in `dtype`."""
    n = int(np.prod(state["shape"], dtype=np.int64))
    bs = int(state["blocksize"])
    if bs <= 0 or hole.nbytes != (n + 1) // 2 or plug.nbytes != hole.nbytes or am.nbytes != 4 * ((n + bs - 1) // bs):
        raise ValueError(f"module planes do not match its state {state}")
    if dtype == "BF16":
        out = np.empty(n, dtype="<u2")
        fn = lib.glint_expand_packed_to_bf16_host
    else:
        out = np.empty(n, dtype="<f4")
        fn = lib.glint_expand_packed_to_f32_host
    if n:
        rc = fn(hole.ctypes.data, plug.ctypes.data, am.ctypes.data, n, bs, out.ctypes.data)
        if rc != 0:
            raise RuntimeError(f"{fn.__name__} rc={rc}")
    return out.astype("<f2") if dtype == "F16" else out


def unpin(pin_dir: Path, out: Path, dtype: str = "BF16") -> dict:
    """As glint_unpin.unpin (glint_unpin.py:44-88)."""
    if dtype not in DTYPES:
        raise ValueError(f"dtype must be one of {DTYPES}")
    root = Path(pin_dir).expanduser().resolve()
    pj = root / "pin.json"
    if not pj.is_file():
        raise FileNotFoundError(f"no pin.json in {root}")
    meta = json.loads(pj.read_text())
    if meta.get("schema") != "glint_pin_v1":
        raise ValueError(f"not a glint_pin_v1 pin: {meta.get('schema')}")
    index = root / INDEX_NAME
    shard_names = (sorted(set(json.loads(index.read_text())["weight_map"].values())) if index.is_file()
                   else ["model.safetensors"])
    out = Path(out).expanduser().resolve()
    readers: Dict[str, Reader] = {}
    try:
        for s in shard_names:
            readers[s] = Reader(str(root / s))
        where: Dict[str, Tuple[str, Entry]] = {}
        for s in shard_names:
            for e in readers[s].entries:
                where[e.name] = (s, e)
        stems = [n[: -len(STATE_SUFFIX)] for n in where if n.endswith(STATE_SUFFIX)]
        stem_of = {stem + ".weight": stem for stem in stems}
        owned = {m for stem in stems for m in _module_names(stem)}
        lib = glint_cuda.require_gpu("GLINT expand", "the reference's glint_unpin.py")
        if "_glint_cells" in where:
            s, e = where["_glint_cells"]
            compiled = np.empty(256, dtype="<f4")
            lib.glint_cells_f32(compiled.ctypes.data)
            if readers[s].view(e).tobytes() != compiled.tobytes():
                raise RuntimeError("the pin's _glint_cells differs from the codebook compiled into the kernels; "
                                   "the reference's glint_unpin.py expands with a pin's own table")

        def view(name: str) -> np.ndarray:
            s, e = where[name]
            return readers[s].view(e)

        # each output shard's entries, in the pin's order, sizes known up front
        plan: Dict[str, List[Tuple[str, str, Tuple[int, ...], int, Optional[str]]]] = {s: [] for s in shard_names}
        for name, (s, e) in where.items():
            if name in stem_of:
                state = json.loads(view(stem_of[name] + STATE_SUFFIX).tobytes().decode())
                shape = tuple(int(d) for d in state["shape"])
                n = int(np.prod(shape, dtype=np.int64))
                plan[s].append((name, dtype, shape, n * _WIDTH[dtype], stem_of[name]))
            elif name not in owned and name != "_glint_cells":
                plan[s].append((name, e.dtype, e.shape, e.nbytes, None))
        out.mkdir(parents=True, exist_ok=True)
        weight_map: Dict[str, str] = {}
        total = 0
        n_expanded = 0
        for s in shard_names:
            entries = plan[s]
            wt = ThreadedWriter(Writer(str(out / s), [(n, d, sh, nb) for n, d, sh, nb, _ in entries],
                                     {"format": "pt", "unpinned_from": "glint"}))
            ok = False
            try:
                for k, (name, _d, _sh, _nb, stem) in enumerate(entries):
                    if stem is None:
                        wt.put(k, name, view(name))
                        continue
                    w, p, a, st = _module_names(stem)
                    state = json.loads(view(st).tobytes().decode())
                    wt.put(k, name, _expand(lib, state, view(w), view(p), view(a), dtype))
                    n_expanded += 1
                ok = True
            finally:
                wt.finish(abort=not ok)
            for name, _d, _sh, nbytes, _ in entries:
                weight_map[name] = s
                total += nbytes
        if len(shard_names) > 1:
            (out / INDEX_NAME).write_text(
                json.dumps({"metadata": {"total_size": total}, "weight_map": weight_map}, indent=2) + "\n")
        for side in meta.get("sidecar", []):
            p = root / side
            if p.is_file():
                shutil.copyfile(p, out / side)
    finally:
        for r in readers.values():
            r.close()
    return {"out": str(out), "dtype": dtype, "n_expanded": n_expanded, "shards": list(shard_names)}


def main(argv: Optional[List[str]] = None) -> int:
    p = argparse.ArgumentParser(description="GLINT pin -> dense safetensors, expanded on the GPU")
    p.add_argument("--pin", required=True)
    p.add_argument("--out", required=True)
    p.add_argument("--dtype", default="BF16", choices=DTYPES)
    args = p.parse_args(argv)
    print(json.dumps(unpin(Path(args.pin), Path(args.out), args.dtype), indent=2))
    return 0


if __name__ == "__main__":
    sys.exit(main())
