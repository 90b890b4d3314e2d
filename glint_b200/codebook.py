"""GLINT codebook generator: GLINT_CELLS[hole][plug] from the 16 parent centres.

Restates the reference's offline generator (Jadon-Fox/glint glint_codec.py:60-113,
build_cells; glint_codec.py:162-172, write_c_header), which produced the table
that every kernel of this library carries (include/glint_cells.h):

  1. Voronoi cells of the parents on [-1, 1]: the bounds are -1, the midpoints of
     neighbouring parents, and 1 (glint_codec.py:87-92).
  2. Each cell [lo, hi] is cut into 16 children of equal probability mass under a
     normal law of standard deviation 1/3 (glint_codec.py:93-106): with
     p0 = Phi(3 lo) and p1 = Phi(3 hi) (p1 forced above p0 by 1e-12 if the cell
     carries no mass in f64), child i sits at Phi^-1(p0 + (p1 - p0)(i + 1/2)/16) / 3,
     clamped into [lo, hi].
  3. Phi is 0.5 (1 + erf(x / sqrt 2)); Phi^-1 is P. J. Acklam's rational
     approximation of the inverse normal distribution function ("An algorithm for
     computing the inverse normal cumulative distribution function", 2003): a
     central rational function for 0.02425 <= p <= 0.97575 and tail forms in
     sqrt(-2 ln p) outside, with the coefficients the reference carries.  The
     reference evaluates the same polynomials in Horner form, and so does this
     module, so the f64 children (and therefore the f32 table) come out the same
     bit for bit.  Measured against scipy's inverse: relative error <= 1.13e-9 in
     the tails (Acklam's stated bound), but up to 2.8e-5 at the edges of the
     central region (1e-6 on 0.1 <= p <= 0.9), so the children sit within 0.23 %
     of a bin's mass of the exact equal-mass points.  The table is data and must
     equal the reference's, so this is kept as it is.

The parents themselves are data (the NF4 geometry) and come from the library's
header, so the generator and the kernels read one table.
"""
from __future__ import annotations

import math
import re
from pathlib import Path
from typing import List, Sequence

import numpy as np

HEADER = Path(__file__).resolve().parents[1] / "include" / "glint_cells.h"
CHILDREN = 16
SIGMA_INV = 3.0  # the children follow N(0, 1/3) inside every parent cell

# Acklam's coefficients: central numerator / denominator, tail numerator / denominator
_A = (-3.969683028665376e01, 2.209460984245205e02, -2.759285104469687e02, 1.383577459574091e02,
      -3.066479806614736e01, 2.506628277459239e00)
_B = (-5.447609879822406e01, 1.615858368580409e02, -1.556989798598866e02, 6.680131188771972e01,
      -1.328068155288572e01, 1.0)
_C = (-7.784894002430293e-03, -3.223964580411365e-01, -2.400758277161838e00, -2.549732539343734e00,
      4.374664141464968e00, 2.938163982698783e00)
_D = (7.784695709041462e-03, 3.224671290700398e-01, 2.445134137142996e00, 3.754408661907416e00, 1.0)
_P_LOW = 0.02425


def _horner(coef: Sequence[float], t: float) -> float:
    """coef[0] t^(n-1) + ... + coef[n-1], evaluated as (((c0 t + c1) t + c2) ...)."""
    acc = coef[0]
    for c in coef[1:]:
        acc = acc * t + c
    return acc


def norm_cdf(x: float) -> float:
    """Phi(x) of the standard normal law."""
    return 0.5 * (1.0 + math.erf(x / math.sqrt(2.0)))


def norm_ppf(p: float) -> float:
    """Acklam's inverse of Phi; +-1e9 outside (0, 1), as the reference returns."""
    if p <= 0.0:
        return -1e9
    if p >= 1.0:
        return 1e9
    if p < _P_LOW:
        q = math.sqrt(-2.0 * math.log(p))
        return _horner(_C, q) / _horner(_D, q)
    if p > 1.0 - _P_LOW:
        q = math.sqrt(-2.0 * math.log(1.0 - p))
        return -_horner(_C, q) / _horner(_D, q)
    q = p - 0.5
    r = q * q
    return _horner(_A, r) * q / _horner(_B, r)


def _hex_literals(macro: str, text: str) -> List[str]:
    body = re.search(r"#define " + macro + r" \{(.*?)\}\s*\n(?!\s*\{)", text, re.S)
    if body is None:
        raise ValueError(f"{macro} not found in the header")
    return re.findall(r"-?0x[0-9a-f.]+p[-+][0-9]+f", body.group(1))


def parents() -> List[float]:
    """The 16 parent centres (f32 values) as written in include/glint_cells.h."""
    lits = _hex_literals("GLINT_PARENT_INIT", HEADER.read_text())
    if len(lits) != 16:
        raise ValueError("GLINT_PARENT_INIT must hold 16 values")
    return [float.fromhex(s[:-1]) for s in lits]


def voronoi_bounds(parent: Sequence[float] | None = None) -> List[float]:
    """-1, the midpoints of neighbouring parents, 1 (17 bounds of 16 cells)."""
    p = list(parents() if parent is None else parent)
    return [-1.0] + [0.5 * (p[i] + p[i + 1]) for i in range(len(p) - 1)] + [1.0]


def children(lo: float, hi: float, n: int = CHILDREN) -> List[float]:
    """n equal-mass children of the cell [lo, hi] under N(0, 1/3), ascending."""
    p0 = norm_cdf(lo * SIGMA_INV)
    p1 = norm_cdf(hi * SIGMA_INV)
    if p1 <= p0:
        p1 = p0 + 1e-12
    out = []
    for i in range(n):
        z = norm_ppf(p0 + (p1 - p0) * (i + 0.5) / n) / SIGMA_INV
        out.append(min(max(z, lo), hi))
    return out


def build_cells(parent: Sequence[float] | None = None) -> List[List[float]]:
    """CELLS[hole][plug] in f64: row h holds the 16 children of parent h."""
    b = voronoi_bounds(parent)
    return [children(b[k], b[k + 1]) for k in range(len(b) - 1)]


def cells_f32(cells: List[List[float]] | None = None) -> np.ndarray:
    """The table as the kernels hold it: f32 [16, 16]."""
    return np.asarray(build_cells() if cells is None else cells, dtype=np.float64).astype(np.float32)


def write_c_header(path: str, cells: List[List[float]] | None = None) -> None:
    """The reference's header (glint_codec.py:162-172): a static f32 table with
    every value printed to ten significant digits ("%.9e" with an f suffix), which
    a C compiler rounds back to the same f32."""
    rows = build_cells() if cells is None else cells
    lines = ["/* Generated by glint_codec.py. GLINT_CELLS[hole][plug]. */",
             "#ifndef GLINT_CELLS_H_", "#define GLINT_CELLS_H_",
             "static const float GLINT_CELLS[16][16] = {"]
    lines += [" { " + ", ".join(f"{float(x):.9e}f" for x in row) + " }," for row in rows]
    lines += ["};", "#endif", ""]
    Path(path).write_text("\n".join(lines), encoding="utf-8")


def hex_literal(v: float) -> str:
    """An f32 value as the exact C99 hexadecimal literal include/glint_cells.h uses
    (six hex digits of mantissa, e.g. -0x1.fb3d6ep-1f; zero as 0x0.0p+0f)."""
    v = float(np.float32(v))
    if v == 0.0:
        return ("-" if math.copysign(1.0, v) < 0 else "") + "0x0.0p+0f"
    h = v.hex()  # [-]0x1.<13 hex digits>p<exp>: an f32 mantissa ends after 6 digits
    sign, rest = ("-", h[1:]) if h[0] == "-" else ("", h)
    mant, exp = rest[2:].split("p")
    lead, frac = mant.split(".")
    if frac[6:].strip("0"):
        raise ValueError(f"{v!r} is not an f32 value")
    return f"{sign}0x{lead}.{frac[:6]}p{'+' if not exp.startswith('-') else ''}{exp.lstrip('+')}f"


def header_literals() -> List[str]:
    """GLINT_CELLS_INIT of include/glint_cells.h, value by value."""
    return _hex_literals("GLINT_CELLS_INIT", HEADER.read_text())
