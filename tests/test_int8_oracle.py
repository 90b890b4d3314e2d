"""The INT8 W8A8 oracle (oracle/glint_oracle.c, restating cuda/int8_mma_gemm.cu of the
reference) against direct numpy statements of its rules: the activation quantization
(s = amax / 127, rint, clamp), the res4 nibble decode and the per-block scaled sums.
On the GPU (tests/test_gpu_int8.py) it is checked against that file itself, built
unchanged for sm_100a."""
import sys
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[1]
sys.path.insert(0, str(ROOT / "oracle"))

import glint_oracle as O  # noqa: E402


def _x(m, k, seed, scale=1.0):
    return O.f32_to_bf16((np.random.default_rng(seed).normal(0, scale, m * k)).astype(np.float32))


def test_quant_rule():
    m, k = 5, 192
    x = _x(m, k, 1)
    x[:64] = 0  # an all-zero block: scale 1, codes 0
    q, s = O.int8_quant(x, m, k)
    xf = O.bf16_to_f32(x).reshape(m, k // 64, 64)
    am = np.abs(xf).max(axis=2)
    want_s = np.where(am > 0, (am / np.float32(127)).astype(np.float32), np.float32(1)).astype(np.float32)
    assert np.array_equal(s.reshape(m, k // 64).view(np.uint32), want_s.view(np.uint32))
    want_q = np.clip(np.rint(xf / want_s[:, :, None]), -127, 127).astype(np.int8).reshape(-1)
    assert np.array_equal(q, want_q)
    assert s[0] == 1.0 and not q[:64].any()


def test_residual_pass_shrinks_the_error():
    m, k = 3, 256
    x = _x(m, k, 2)
    q, s = O.int8_quant(x, m, k)
    rq, rs = O.int8_quant(x, m, k, prev=(q, s))
    xf = O.bf16_to_f32(x).astype(np.float64).reshape(m, k // 64, 64)
    one = q.reshape(m, k // 64, 64) * s.reshape(m, k // 64, 1).astype(np.float64)
    two = one + rq.reshape(m, k // 64, 64) * rs.reshape(m, k // 64, 1).astype(np.float64)
    assert np.abs(xf - two).max() < np.abs(xf - one).max() / 50


def _weights(n, k, seed):
    wq, ws = O.int8_quant(_x(n, k, seed, 0.02), n, k)  # the pin rule: 64 consecutive weights per scale
    return wq, ws


def test_gemm_is_the_scaled_block_sum():
    m, n, k = 4, 24, 192
    xq, sx = O.int8_quant(_x(m, k, 3), m, k)
    wq, ws = _weights(n, k, 4)
    y = O.int8_gemm(xq, sx, wq, ws, m, n, k)
    xd = xq.reshape(m, k // 64, 64).astype(np.int64)
    wd = wq.reshape(n, k // 64, 64).astype(np.int64)
    dots = np.einsum("mbj,nbj->mnb", xd, wd)  # exact int32 block sums
    ref = (dots * sx.reshape(m, 1, k // 64) * ws.reshape(1, n, k // 64)).sum(axis=2)
    assert np.abs(y - ref).max() <= 1e-6 * max(1.0, np.abs(ref).max())
    # accumulate adds onto y
    y2 = O.int8_gemm(xq, sx, wq, ws, m, n, k, y=y, accumulate=True)
    assert np.allclose(y2, 2 * y, rtol=1e-6)


def test_res4_plug_decode():
    """nibble - 8 with element 2i in the low nibble, its own per-64 scale; fused = base + plug."""
    m, n, k = 2, 16, 128
    xq, sx = O.int8_quant(_x(m, k, 5), m, k)
    wq, ws = _weights(n, k, 6)
    rng = np.random.default_rng(7)
    q4 = rng.integers(0, 256, n * k // 2, dtype=np.uint8)
    ps = (rng.random(n * k // 64) * 1e-3).astype(np.float32)
    fused = O.int8_gemm(xq, sx, wq, ws, m, n, k, plug=(q4, ps))
    nib = np.stack([q4 & 15, q4 >> 4], axis=1).reshape(-1).astype(np.int8) - 8
    base = O.int8_gemm(xq, sx, wq, ws, m, n, k)
    plug_only = O.int8_gemm(xq, sx, nib, ps, m, n, k)
    assert np.allclose(fused, base + plug_only, rtol=1e-5, atol=1e-7)
    assert nib.min() >= -8 and nib.max() <= 7
