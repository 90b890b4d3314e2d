"""Pin and unpin pipelines (glint_b200/pin.py, glint_b200/unpin.py, glint_b200/st_io.py)
against the files the reference's own tools wrote (tests/golden/pin/, made by
tests/golden/make_pin_golden.py with glint_pin.convert and glint_unpin.unpin of
Jadon-Fox/glint).

CPU: the safetensors writer reproduces every reference-written file byte for byte
from its tensors; the plan (which tensors are linears) equals the reference's dry
run; without a usable GPU the product refuses instead of encoding on the host.
GPU: the whole conversion of the two-shard model and of the one-file model gives the
reference's shard files, index and sidecars byte for byte, pin.json and
CONVERT_REPORT.json with the same fields, and per-linear rmse within 1e-9 relative
(both sum squares in f64, in different orders); a multi-chunk tensor's planes equal
the oracle's encode; unpin of the reference's pins to BF16, F16 and F32 gives the
reference unpin's files byte for byte and its return value.
"""
import filecmp
import json
import math
import shutil
import sys
from pathlib import Path

import numpy as np
import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from glint_b200 import glint_cuda, pin, unpin
from glint_b200.st_io import Reader, Writer, header_bytes, write_file

GOLD = Path(__file__).resolve().parent / "golden" / "pin"
CASES = [(GOLD / "src", GOLD / "ref"), (GOLD / "single.safetensors", GOLD / "ref_single")]


def _tensors(path):
    with Reader(str(path)) as r:
        return r.metadata, [(e.name, e.dtype, e.shape, r.view(e).tobytes()) for e in r.entries]


@pytest.mark.parametrize("rel", ["src/model-00001-of-00002.safetensors", "src/model-00002-of-00002.safetensors",
                                 "ref/model-00001-of-00002.safetensors", "ref/model-00002-of-00002.safetensors",
                                 "ref_single/model.safetensors", "single.safetensors"])
def test_writer_reproduces_reference_files(rel, tmp_path):
    meta, tensors = _tensors(GOLD / rel)
    write_file(str(tmp_path / "x.safetensors"), tensors, meta)
    assert (tmp_path / "x.safetensors").read_bytes() == (GOLD / rel).read_bytes()


_DT = ["BOOL", "U8", "I8", "I16", "U16", "F16", "BF16", "I32", "U32", "F32", "F64", "I64", "U64"]


@settings(max_examples=60, deadline=None)
@given(spec=st.lists(st.tuples(st.sampled_from(_DT), st.lists(st.integers(0, 5), min_size=0, max_size=3)),
                     min_size=0, max_size=6),
       meta=st.dictionaries(st.text("abcxyz", min_size=1, max_size=4), st.text(max_size=6), max_size=2),
       seed=st.integers(0, 2 ** 16))
def test_write_read_round_trip(spec, meta, seed, tmp_path_factory):
    """Any dtypes, shapes (empty ones too) and metadata: the reader gets back the
    names, dtypes, shapes, metadata and bytes the writer was given, with the data
    starting on an 8-byte boundary."""
    from glint_b200.st_io import DTYPE_WIDTH
    rng = np.random.default_rng(seed)
    tensors = []
    for i, (dt, shape) in enumerate(spec):
        nbytes = int(np.prod(shape, dtype=np.int64)) * DTYPE_WIDTH[dt]
        tensors.append((f"t{i}.{dt.lower()}", dt, tuple(shape), rng.integers(0, 256, nbytes, dtype=np.uint8).tobytes()))
    path = tmp_path_factory.mktemp("rt") / "x.safetensors"
    write_file(str(path), tensors, meta)
    got_meta, got = _tensors(path)
    assert got_meta == meta
    assert [(n, d, tuple(sh), b) for n, d, sh, b in got] == tensors
    with Reader(str(path)) as r:
        assert r.data_start % 8 == 0


def test_header_padding_and_order():
    hb = header_bytes([("b", "U8", (3,), 3), ("a", "F32", (1,), 4)], {"format": "pt"})
    assert len(hb) % 8 == 0
    head = json.loads(hb[8:].decode())
    assert list(head) == ["__metadata__", "b", "a"]
    assert head["a"]["data_offsets"] == [3, 7]


def test_positional_writes_in_any_order_and_threads(tmp_path):
    """put_at from several threads in reverse order gives the reference's bytes."""
    import threading
    rel = "ref/model-00001-of-00002.safetensors"
    meta, tensors = _tensors(GOLD / rel)
    w = Writer(str(tmp_path / "x.safetensors"), [(n, d, s, len(b)) for n, d, s, b in tensors], meta)
    order = list(range(len(tensors)))[::-1]
    th = [threading.Thread(target=lambda ks: [w.put_at(k, tensors[k][0], tensors[k][3]) for k in ks],
                           args=(order[j::3],)) for j in range(3)]
    for t in th:
        t.start()
    for t in th:
        t.join()
    with pytest.raises(ValueError):
        w.put_at(0, tensors[0][0], tensors[0][3])  # twice
    w.close()
    assert (tmp_path / "x.safetensors").read_bytes() == (GOLD / rel).read_bytes()


def test_writer_checks_order_and_sizes(tmp_path):
    w = Writer(str(tmp_path / "x.safetensors"), [("a", "U8", (2,), 2), ("b", "U8", (1,), 1)])
    with pytest.raises(ValueError):
        w.put("b", b"\x00")
    w.put("a", b"\x00\x01")
    with pytest.raises(ValueError):
        w.put("b", b"\x00\x01")
    with pytest.raises(ValueError):
        w.close()


@pytest.mark.parametrize("src,ref", CASES)
def test_dry_run_plan_matches_reference(src, ref):
    got = pin.convert(src, Path("unused"), 64, dry_run=True)
    want = json.loads((ref / "dry_run.json").read_text())
    for k in ("schema", "n_linears", "n_keep", "blocksize", "shards", "linears"):
        assert got[k] == want[k], k


def test_resolve_shards_rules(tmp_path):
    with pytest.raises(FileNotFoundError):
        pin.resolve_shards(tmp_path)  # no shard at all
    shutil.copy(GOLD / "single.safetensors", tmp_path / "a.safetensors")
    assert pin.resolve_shards(tmp_path) == [(tmp_path / "a.safetensors").resolve()]
    assert [p.name for p in pin.resolve_shards(GOLD / "src")] == ["model-00001-of-00002.safetensors",
                                                                 "model-00002-of-00002.safetensors"]


def test_no_host_encoder_without_gpu(tmp_path):
    if glint_cuda.gpu_ok():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA"):
        pin.convert(GOLD / "src", tmp_path / "out", 64, allow_cpu=True)
    assert not (tmp_path / "out").exists()


def _same_report(got: dict, want: dict):
    for k in want:
        if k in ("src", "backend", "backends", "rmse_mean", "rmse_max"):
            continue
        assert got[k] == want[k], k
    for k in ("rmse_mean", "rmse_max"):
        assert math.isclose(got[k], want[k], rel_tol=1e-9), (k, got[k], want[k])


@pytest.mark.gpu
@pytest.mark.parametrize("src,ref", CASES)
def test_convert_matches_reference_pin(src, ref, tmp_path):
    out = tmp_path / "pin"
    got = pin.convert(src, out, 64)
    names = sorted(p.name for p in ref.iterdir() if p.name != "dry_run.json")
    assert sorted(p.name for p in out.iterdir()) == names
    for name in names:
        if name.endswith(".json") and name in ("pin.json", "CONVERT_REPORT.json"):
            continue
        assert filecmp.cmp(out / name, ref / name, shallow=False), name
    want = json.loads((ref / "CONVERT_REPORT.json").read_text())
    _same_report(json.loads((out / "pin.json").read_text()), want["pin"])
    _same_report(got["pin"], want["pin"])
    assert got["pin"]["src"] == str(Path(src).resolve())
    assert len(got["modules"]) == len(want["modules"])
    for g, w in zip(got["modules"], want["modules"]):
        assert (g["src"], g["shape"], g["shard"]) == (w["src"], w["shape"], w["shard"])
        assert math.isclose(g["rmse"], w["rmse"], rel_tol=1e-9, abs_tol=0.0), (g, w)
        assert g["backend"] == ("cuda_bf16" if json.loads(
            _state_of(out, g)).get("src_dtype") == "BF16" else "cuda_f32")


def _state_of(out: Path, module: dict) -> bytes:
    with Reader(str(out / module["shard"])) as r:
        e = next(e for e in r.entries if e.name == module["src"] + ".weight.glint_state")
        return r.view(e).tobytes()


@pytest.mark.gpu
def test_convert_multi_chunk_tensor_vs_oracle(tmp_path):
    """A 4096 x 4096 BF16 linear (16.8 M weights, eight pipeline chunks) and a 3 x 5 one:
    planes and absmax byte-equal to the oracle's encode; rmse equal to the f64 rmse of
    the oracle's expand within 1e-9."""
    sys.path.insert(0, str(Path(__file__).resolve().parent.parent / "oracle"))
    import glint_oracle as O
    rng = np.random.default_rng(5)
    w = rng.normal(0, 0.02, 4096 * 4096).astype(np.float32)
    w[rng.choice(w.size, 4096, replace=False)] *= 20
    bits = O.f32_to_bf16(w)
    small = O.f32_to_bf16(rng.normal(0, 1, 15).astype(np.float32))
    src = tmp_path / "m.safetensors"
    write_file(str(src), [("big.weight", "BF16", (4096, 4096), bits.tobytes()),
                          ("small.weight", "BF16", (3, 5), small.tobytes())])
    got = pin.convert(src, tmp_path / "pin", 64)
    _, out = _tensors(tmp_path / "pin" / "model.safetensors")
    by = {n: b for n, _d, _s, b in out}
    for name, b, n in (("big", bits, 4096 * 4096), ("small", small, 15)):
        ho, po, ao = O.encode_bf16(b, 64)
        assert by[name + ".weight"] == ho.tobytes()
        assert by[name + ".weight.glint_plug"] == po.tobytes()
        assert by[name + ".weight.absmax"] == ao.astype("<f4").tobytes()
        ref = O.expand_f32(ho, po, ao, n, 64).astype(np.float64)
        d = O.bf16_to_f32(b).astype(np.float64) - ref
        want = float(np.sqrt(np.mean(d * d)))
        mod = next(m for m in got["modules"] if m["src"] == name)
        assert math.isclose(mod["rmse"], want, rel_tol=1e-9), (mod["rmse"], want)


UNPIN_CASES = [(GOLD / "ref", GOLD / "unpin_bf16", "BF16"), (GOLD / "ref_single", GOLD / "unpin_single_bf16", "BF16"),
               (GOLD / "ref_single", GOLD / "unpin_single_f16", "F16"),
               (GOLD / "ref_single", GOLD / "unpin_single_f32", "F32")]


def test_unpin_argument_errors(tmp_path):
    with pytest.raises(ValueError):
        unpin.unpin(GOLD / "ref", tmp_path / "o", "F64")
    with pytest.raises(FileNotFoundError):
        unpin.unpin(tmp_path, tmp_path / "o")
    bad = tmp_path / "bad"
    shutil.copytree(GOLD / "ref_single", bad)
    doc = json.loads((bad / "pin.json").read_text())
    doc["schema"] = "something_else"
    (bad / "pin.json").write_text(json.dumps(doc))
    with pytest.raises(ValueError, match="glint_pin_v1"):
        unpin.unpin(bad, tmp_path / "o")


def test_unpin_no_host_path_without_gpu(tmp_path):
    if glint_cuda.gpu_ok():
        pytest.skip("a GPU is present")
    with pytest.raises(RuntimeError, match="CUDA"):
        unpin.unpin(GOLD / "ref", tmp_path / "o")
    assert not (tmp_path / "o").exists()


@pytest.mark.gpu
@pytest.mark.parametrize("pin_dir,ref,dtype", UNPIN_CASES)
def test_unpin_matches_reference(pin_dir, ref, dtype, tmp_path):
    out = tmp_path / "dense"
    got = unpin.unpin(pin_dir, out, dtype)
    want = json.loads((ref / "unpin.json").read_text())
    assert got["out"] == str(out.resolve())
    got["out"] = want["out"]
    assert got == want
    names = sorted(p.name for p in ref.iterdir() if p.name != "unpin.json")
    assert sorted(p.name for p in out.iterdir()) == names
    for name in names:
        assert filecmp.cmp(out / name, ref / name, shallow=False), name


@pytest.mark.gpu
def test_unpin_refuses_a_foreign_codebook(tmp_path):
    """A pin whose _glint_cells is not the compiled table: refused, not expanded wrongly."""
    foreign = tmp_path / "pin"
    shutil.copytree(GOLD / "ref_single", foreign)
    meta, tensors = _tensors(foreign / "model.safetensors")
    tensors = [(n, d, s, (np.frombuffer(b, "<f4") * np.float32(2)).tobytes() if n == "_glint_cells" else b)
               for n, d, s, b in tensors]
    write_file(str(foreign / "model.safetensors"), tensors, meta)
    with pytest.raises(RuntimeError, match="_glint_cells"):
        unpin.unpin(foreign, tmp_path / "o")
