"""The codebook generator (glint_b200/codebook.py) against the reference's own
generator (glint_codec.py:87-113, 162-172; fixture tests/golden/codebook.json,
written by tests/golden/make_codebook_golden.py) and against the table every
kernel of this library carries (include/glint_cells.h)."""
import json
import math
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT))

from glint_b200 import codebook as C  # noqa: E402

GOLD = json.loads((ROOT / "tests" / "golden" / "codebook.json").read_text())
TABLES = json.loads((ROOT / "tests" / "golden" / "tables.json").read_text())


def test_voronoi_bounds_match_reference_bit_for_bit():
    assert [b.hex() for b in C.voronoi_bounds()] == GOLD["voronoi_hex"]


def test_children_match_reference_bit_for_bit():
    mine = [v.hex() for row in C.build_cells() for v in row]
    assert mine == GOLD["cells_hex"]


def test_f32_table_is_the_library_table():
    """f32 of the generated children == the pinned reference table and the
    literals of include/glint_cells.h, value for value."""
    bits = C.cells_f32().reshape(-1).view(np.uint32)
    assert [int(b) for b in bits] == TABLES["cells_bits"]
    assert [C.hex_literal(v) for v in C.cells_f32().reshape(-1)] == C.header_literals()
    assert [int(b) for b in np.asarray(C.parents(), np.float32).view(np.uint32)] == TABLES["parent_bits"]


def test_header_text_matches_reference(tmp_path):
    p = tmp_path / "glint_cells.h"
    C.write_c_header(str(p))
    assert p.read_text(encoding="utf-8") == GOLD["header_text"]


def test_header_decimal_literals_round_trip_to_the_table(tmp_path):
    """The ten-digit literals a C compiler reads back are the same f32 values."""
    import re
    p = tmp_path / "glint_cells.h"
    C.write_c_header(str(p))
    nums = re.findall(r"[-+0-9.]+e[-+][0-9]+f", p.read_text())
    assert len(nums) == 256
    got = np.asarray([float(x[:-1]) for x in nums], np.float32)
    assert np.array_equal(got.view(np.uint32), C.cells_f32().reshape(-1).view(np.uint32))


def test_table_geometry():
    """Every child lies in its parent's Voronoi cell, rows ascend, the whole table
    ascends strictly, and the children split each cell's N(0, 1/3) mass evenly."""
    b = C.voronoi_bounds()
    cells = C.build_cells()
    flat = [v for row in cells for v in row]
    assert all(x < y for x, y in zip(flat, flat[1:]))
    for k, row in enumerate(cells):
        assert all(b[k] <= v <= b[k + 1] for v in row)
        p0, p1 = C.norm_cdf(3 * b[k]), C.norm_cdf(3 * b[k + 1])
        for i, v in enumerate(row):
            # within 0.5 % of one child's mass of the exact equal-mass point (the
            # reference's inverse normal is good to 2.8e-5 relative; 0.23 % seen)
            want = p0 + (p1 - p0) * (i + 0.5) / 16
            assert abs(C.norm_cdf(3 * v) - want) <= 0.005 * (p1 - p0) / 16


def test_norm_ppf_error_profile():
    """Against scipy: the tails meet Acklam's stated 1.15e-9 relative bound; the
    central form with the reference's coefficients is good to 3e-5 at its edges
    and 1e-6 on [0.1, 0.9] (the children above are pinned bit for bit anyway)."""
    stats = pytest.importorskip("scipy.stats")
    tails = np.concatenate([np.geomspace(1e-12, 0.0242, 200), 1.0 - np.geomspace(1e-12, 0.0242, 200)])
    for p in tails:
        want = float(stats.norm.ppf(p))
        assert abs(C.norm_ppf(float(p)) - want) <= 1.15e-9 * abs(want), p
    for p in np.linspace(0.02425, 0.97575, 401):
        want = float(stats.norm.ppf(p))
        bound = 1e-6 if 0.1 <= p <= 0.9 else 3e-5
        assert abs(C.norm_ppf(float(p)) - want) <= bound * abs(want) + 1e-15, p
    assert C.norm_ppf(0.0) == -1e9 and C.norm_ppf(1.0) == 1e9


def test_degenerate_cell_guard():
    """A cell with no f64 mass (both bounds deep in one tail) still yields 16
    clamped children, as the reference's p1 = p0 + 1e-12 guard gives."""
    out = C.children(9.0, 9.5)
    assert len(out) == 16 and all(9.0 <= v <= 9.5 for v in out)
    assert not any(math.isnan(v) for v in out)
