"""The CPU oracle (oracle/glint_oracle.c) against the reference's own outputs.

tests/golden/*.npz were written by tests/golden/make_golden.py, which ran the
reference's glint_np.py / glint_htile_sim.py.  A mismatch here means the oracle
no longer restates the reference and every GPU parity result built on it is void.
"""
import json
from pathlib import Path

import numpy as np
import pytest

import glint_oracle as O

G = Path(__file__).resolve().parent / "golden"


def _cases(npz):
    d = np.load(G / npz)
    names = sorted({k.split("__")[0] for k in d.files})
    return d, names


def test_tables_match_reference_codebook():
    """include/glint_cells.h == glint_codec.CELLS / PARENT as f32 bits
    (reference test_glint_tools.py:38-50 checks the same sync)."""
    import re
    t = json.loads((G / "tables.json").read_text())
    hdr = (G.parent.parent / "include" / "glint_cells.h").read_text()
    lits = re.findall(r"(-?0x[0-9a-f.]+p[-+]?\d+)f", hdr)
    vals = np.array([float.fromhex(x) for x in lits], np.float32).view(np.uint32)
    assert vals.size == 256 + 16
    assert vals[:256].tolist() == t["cells_bits"]
    assert vals[256:].tolist() == t["parent_bits"]
    cells = vals[:256].view(np.float32)
    assert np.all(np.diff(cells) > 0), "flattened codebook must be strictly ascending"


@pytest.mark.parametrize("name", _cases("encode_bf16.npz")[1])
def test_oracle_encode_bf16_matches_reference(name):
    d = np.load(G / "encode_bf16.npz")
    bs = int(d[name + "__bs"][0])
    h, p, am = O.encode_bf16(d[name + "__w"], bs)
    assert h.tobytes() == d[name + "__hole"].tobytes()
    assert p.tobytes() == d[name + "__plug"].tobytes()
    assert am.tobytes() == d[name + "__absmax"].tobytes()
    n = d[name + "__w"].size
    assert O.expand_f32(h, p, am, n, bs).tobytes() == d[name + "__expand_f32"].tobytes()
    assert O.expand_bf16(h, p, am, n, bs).tobytes() == d[name + "__expand_bf16"].tobytes()


@pytest.mark.parametrize("name", _cases("encode_f32.npz")[1])
def test_oracle_encode_f32_matches_reference(name):
    d = np.load(G / "encode_f32.npz")
    bs = int(d[name + "__bs"][0])
    h, p, am = O.encode_f32(d[name + "__w"], bs)
    assert h.tobytes() == d[name + "__hole"].tobytes()
    assert p.tobytes() == d[name + "__plug"].tobytes()
    assert am.tobytes() == d[name + "__absmax"].tobytes()


def test_oracle_expand_specials_match_reference():
    d = np.load(G / "expand.npz")
    n, bs = int(d["n"][0]), int(d["bs"][0])
    assert O.expand_f32(d["hole"], d["plug"], d["absmax"], n, bs).tobytes() == d["expand_f32"].tobytes()
    assert O.expand_bf16(d["hole"], d["plug"], d["absmax"], n, bs).tobytes() == d["expand_bf16"].tobytes()


@pytest.mark.parametrize("key", _cases("htile.npz")[1])
def test_oracle_htile_matches_reference_sim(key):
    d = np.load(G / "htile.npz")
    M, N, K, bs = (int(v) for v in d[key + "__shape"])
    y = O.htile(d[key + "__hole"], d[key + "__plug"], d[key + "__absmax"], d[key + "__x"], M, N, K, bs)
    ref = d[key + "__y"].reshape(M, N)
    # both sum f32 products in f64; only the final f32 rounding differs
    assert np.max(np.abs(y - ref) / (1 + np.abs(ref))) < 1e-6


def test_oracle_bf16_rounding_rule():
    """RNE ties and the NaN rule (reference test_glint_tools.py:31-37, glint_np.py:25-31)."""
    one, ulp = 1.0, 2.0 ** -7
    v = np.array([one + ulp / 2, one + 1.5 * ulp, one + 0.75 * ulp, -(one + ulp / 2), np.nan], np.float32)
    b = O.f32_to_bf16(v)
    assert O.bf16_to_f32(b[:4]).tolist() == [one, one + 2 * ulp, one + ulp, -one]
    assert np.isnan(O.bf16_to_f32(b[4:5]))[0]
    L = O.lib()
    assert [L.orc_f32_to_bf16(float(x)) for x in v[:4]] == b[:4].tolist()
