"""Arithmetic identities the encode kernel relies on, checked exhaustively on the
CPU with IEEE f32 (numpy)."""
import numpy as np


def _f32(bits):
    return np.array(bits, dtype=np.uint32).view(np.float32)


def _bits(x):
    return np.asarray(x, dtype=np.float32).view(np.uint32).astype(np.int64)


def test_block_reciprocal_table_is_correctly_rounded():
    """encode.cu block_rcp: for a BF16-valued block scale s = 1.k x 2^E in the
    Markstein range [2^-60, 2^60], RN(1/s) equals the entry RN(1/1.k) of a
    128-entry table with 127 - E added to its exponent field."""
    k = np.arange(128)
    tab = _bits(np.float32(1) / (np.float32(1) + k.astype(np.float32) / np.float32(128)))
    E = np.arange(127 - 60, 127 + 61)
    sb = (E[:, None] << 23) | (k[None, :] << 16)
    s = _f32(sb.ravel())
    keep = (s >= np.float32(2.0 ** -60)) & (s <= np.float32(2.0 ** 60))
    got = tab[(sb.ravel() >> 16) & 0x7F] + (127 << 23) - (sb.ravel() & 0x7F800000)
    ref = _bits(np.float32(1) / s)
    assert keep.sum() > 15000
    assert np.array_equal(got[keep], ref[keep])


def test_lowered_threshold_sign_rule():
    """encode.cu codes16: with thr' the float just below thr, v >= thr exactly when
    the f32 difference thr' - v is negative (sign bit set), for thresholds and
    values around the cell boundaries, signed zeros and the no-threshold +inf."""
    rng = np.random.default_rng(0)
    thr = np.concatenate([rng.uniform(-1, 1, 2000).astype(np.float32),
                          np.float32([2.0 ** -140, -2.0 ** -140, 1e-30, -1e-30, np.inf])])
    tb = _bits(thr)
    prev = np.where(tb >> 31, tb + 1, tb - 1)
    tp = _f32(prev.astype(np.uint32))
    for t, t2 in zip(thr, tp):
        near = _f32((_bits(np.float32(t)) + np.arange(-3, 4)).astype(np.uint32)) if np.isfinite(t) else np.float32([1.0, -1.0])
        v = np.concatenate([near, np.float32([0.0, -0.0, 1.0, -1.0])])
        d = (np.float32(t2) - v).astype(np.float32)
        assert np.array_equal((_bits(d) >> 31) & 1, (v >= t).astype(np.int64)), (t, v)
