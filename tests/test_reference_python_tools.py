"""The reference's own Python tools driving this library unchanged.

oracle/Makefile (target ref-py) stages the reference's Python tools and their test
suite, unmodified, into the git-ignored oracle/_ref/py/.  Here that suite runs with
GLINT_ENCODE_SO pointing at this repository's libglint_encode.so, so its GPU gate
(test_glint_tools.py:215-228: glint_pin.convert through glint_cuda.encode_bf16_cuda,
then glint_verify.verify(parity=True, cuda=True): host re-encode byte parity and
GPU expand within 1e-5) loads and calls this library exactly as it would the
reference's own build.  The two table-sync tests that read the reference's C
sources (include/glint_cells.h, cuda/glint_encode.cu), which are not staged, are
deselected; they concern the reference's files, not this library.

Then the tools' command lines: glint_pin.py converts a two-shard toy model on the
GPU (no --allow-cpu), and glint_verify.py --parity --cuda checks the pin.
"""
import json
import os
import subprocess
import sys
from pathlib import Path

import pytest

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
PY = ROOT / "oracle" / "_ref" / "py"


def _env():
    from glint_b200 import build
    lib = build.build()
    env = dict(os.environ)
    env["GLINT_ENCODE_SO"] = str(lib)
    env["PYTHONPATH"] = str(PY)
    return env


@pytest.fixture(scope="module")
def staged():
    if not (PY / "test_glint_tools.py").is_file():
        pytest.skip("reference Python tools not staged (oracle/Makefile ref-py needs the reference checkout)")
    torch = pytest.importorskip("torch")
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return _env()


def test_reference_tool_suite_gpu_gate_passes_on_this_library(staged):
    r = subprocess.run([sys.executable, "-m", "pytest", "-v", "-p", "no:cacheprovider", "test_glint_tools.py",
                        "test_glint.py", "-k", "not header_in_sync and not parent_table_in_sync"],
                       cwd=PY, env=staged, capture_output=True, text=True, timeout=900)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    # the GPU gate ran (it skips itself when the library does not load or no GPU answers)
    assert "test_cuda_pin_byte_parity_and_expand PASSED" in out, out[-4000:]


def test_reference_pin_and_verify_clis_on_this_library(staged, tmp_path):
    import numpy as np
    sys.path.insert(0, str(PY))
    try:
        from safetensors_io import write_safetensors
    finally:
        sys.path.remove(str(PY))
    rng = np.random.default_rng(5)
    src = tmp_path / "src"
    src.mkdir()

    def bf16(shape):
        w = rng.normal(0, 0.02, int(np.prod(shape))).astype(np.float32)
        u = w.view(np.uint32)
        return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype("<u2").tobytes()
    shards = {"model-00001-of-00002.safetensors": [("model.layers.0.mlp.up_proj.weight", (384, 256)),
                                                   ("model.layers.0.input_layernorm.weight", (256,))],
              "model-00002-of-00002.safetensors": [("model.layers.0.mlp.down_proj.weight", (256, 384)),
                                                   ("model.layers.0.self_attn.q_proj.weight", (256, 256))]}
    weight_map = {}
    for fname, tensors in shards.items():
        write_safetensors(str(src / fname), [(n, "BF16", s, bf16(s)) for n, s in tensors])
        weight_map.update({n: fname for n, _s in tensors})
    (src / "model.safetensors.index.json").write_text(json.dumps({"metadata": {}, "weight_map": weight_map}))
    pin = tmp_path / "pin"
    r = subprocess.run([sys.executable, str(PY / "glint_pin.py"), "--src", str(src), "--out", str(pin)],
                       env=staged, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    report = json.loads((pin / "pin.json").read_text())
    assert "cuda_bf16" in report.get("backends", []), report
    ev = tmp_path / "evidence.json"
    r = subprocess.run([sys.executable, str(PY / "glint_verify.py"), "--pin", str(pin), "--src", str(src), "--parity",
                        "--cuda", "--quiet", "--out", str(ev)], env=staged, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, (r.stdout + r.stderr)[-3000:]
    evidence = json.loads(ev.read_text())
    assert evidence["ok"] is True and evidence["parity_checked"] and evidence["cuda_expand_checked"], evidence
