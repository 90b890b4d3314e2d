"""The K-major decode's oracle (oracle/glint_oracle.c, restating the reference's
Mojo decoders: mojo/p7_glint_select_decode.mojo:120-143, mojo/p7_glint_gemv_km.mojo:17-95,
mojo/p7_select_device.mojo:15-238).  No Mojo toolchain exists here, so the
restatement is pinned by definitions it must satisfy: the layout against a numpy
transpose of the nibbles, the selection against a sort-based statement of its
rule, and parent GEMV + correction over every channel against the H-TILE oracle,
itself pinned to the reference's own golden vectors (test_oracle.py)."""
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))

import glint_oracle as O  # noqa: E402

PARENT = np.array([float.fromhex(s[:-1]) for s in __import__("re").findall(
    r"-?0x[0-9a-f.]+p[-+][0-9]+f",
    (ROOT / "include" / "glint_cells.h").read_text().split("#define GLINT_PARENT_INIT")[1].split("\n")[0])],
    np.float32)


def _weight(n, K, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, n * K).astype(np.float32)
    w[rng.choice(n * K, size=max(1, n * K // 1000), replace=False)] *= np.float32(20)
    return O.encode_bf16(O.f32_to_bf16(w), 64)


def _nibbles(plane, count):
    b = np.asarray(plane, np.uint8)
    return np.stack([b & 15, b >> 4], axis=1).reshape(-1)[:count]


@pytest.mark.parametrize("n,K", [(8, 64), (64, 256), (200, 192)])
def test_kmajor_layout_is_the_nibble_transpose(n, K):
    h, p, a = _weight(n, K, 3)
    hk, pk, sk = O.to_kmajor(h, p, a, n, K)
    for plane, plane_k in ((h, hk), (p, pk)):
        dense = _nibbles(plane, n * K).reshape(n, K)          # [row, channel]
        km = _nibbles(plane_k, n * K).reshape(K, n)           # [channel, row]
        assert np.array_equal(km, dense.T)
    assert np.array_equal(sk.reshape(K // 64, n), a.reshape(n, K // 64).T)


def _select_by_sort(bits, nsel):
    keys = bits.astype(np.int64) & 0x7FFF
    if nsel == 0:
        return np.zeros(0, np.int32)
    if nsel > keys.size:
        return np.arange(keys.size, dtype=np.int32)
    t = np.sort(keys)[::-1][nsel - 1]  # the nsel-th largest key
    return np.nonzero(keys >= t)[0].astype(np.int32)


def test_select_rule_matches_its_sort_definition():
    rng = np.random.default_rng(7)
    x = O.f32_to_bf16(rng.normal(0, 1, 4096).astype(np.float32))
    for nsel in (0, 1, 2, 17, 410, 2048, 4095, 4096, 4097, 100000):
        assert np.array_equal(O.select_topk(x, nsel), _select_by_sort(x, nsel)), nsel


def test_select_ties_specials_and_signs():
    """Ties at the threshold are all kept; |x| ranks by the BF16 magnitude bits, so
    -0 == +0, -inf == +inf, NaN above inf; indices stay ascending."""
    vals = np.array([0.0, -0.0, 1.0, -1.0, 1.0, np.inf, -np.inf, np.nan, 2.0, -2.0, 0.5, 1.0], np.float32)
    x = O.f32_to_bf16(vals)
    for nsel in range(0, 14):
        got = O.select_topk(x, nsel)
        assert np.array_equal(got, _select_by_sort(x, nsel)), nsel
        assert np.all(np.diff(got) > 0)
    assert list(O.select_topk(x, 1)) == [7]              # NaN first
    assert list(O.select_topk(x, 2)) == [5, 6, 7]        # then both infinities (tie)
    # NaN, +-inf, +-2 are the top five; the 6th is a 1.0 and all four +-1.0 are kept
    assert list(O.select_topk(x, 6)) == [2, 3, 4, 5, 6, 7, 8, 9, 11]
    same = O.f32_to_bf16(np.full(300, 0.25, np.float32))
    assert len(O.select_topk(same, 5)) == 300


@pytest.mark.parametrize("n,K", [(64, 256), (256, 1024), (136, 512)])
def test_parent_plus_full_correction_is_htile(n, K):
    h, p, a = _weight(n, K, 11)
    hk, pk, sk = O.to_kmajor(h, p, a, n, K)
    x = O.f32_to_bf16(np.random.default_rng(5).normal(0, 1, K).astype(np.float32))
    y0 = O.gemv_km(hk, sk, x, n, K)
    y = O.apply_corr_k(y0, hk, pk, sk, x, O.select_topk(x, K), n, K)
    ref = O.htile(h, p, a, x, 1, n, K, 64)[0]
    assert np.abs(y - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max())


def test_parent_gemv_against_f64_and_slices():
    n, K = 128, 1024
    h, p, a = _weight(n, K, 13)
    hk, pk, sk = O.to_kmajor(h, p, a, n, K)
    x = O.f32_to_bf16(np.random.default_rng(9).normal(0, 1, K).astype(np.float32))
    hn = _nibbles(h, n * K).reshape(n, K)
    w = PARENT[hn].astype(np.float64) * np.repeat(a.reshape(n, K // 64), 64, axis=1).astype(np.float32)
    ref = w @ O.bf16_to_f32(x).astype(np.float64)
    for ksg in (1, 2, 4, 16):
        y = O.gemv_km(hk, sk, x, n, K, ksg)
        assert np.abs(y - ref).max() <= 1e-5 * max(1.0, np.abs(ref).max()), ksg


def test_partial_selection_is_between():
    """Selecting a subset adds exactly those channels' corrections: the correction
    over a set equals the sum of corrections over a split of it (to f32)."""
    n, K = 64, 512
    h, p, a = _weight(n, K, 17)
    hk, pk, sk = O.to_kmajor(h, p, a, n, K)
    x = O.f32_to_bf16(np.random.default_rng(21).normal(0, 1, K).astype(np.float32))
    sel = O.select_topk(x, 51)
    z = np.zeros(n, np.float32)
    whole = O.apply_corr_k(z, hk, pk, sk, x, sel, n, K)
    parts = O.apply_corr_k(O.apply_corr_k(z, hk, pk, sk, x, sel[:20], n, K), hk, pk, sk, x, sel[20:], n, K)
    assert np.abs(whole - parts).max() <= 1e-5 * max(1.0, np.abs(whole).max())
    assert not np.allclose(whole, 0)
