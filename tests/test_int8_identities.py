"""The two integer/float identities the tcgen05 INT8 kernel (glint_b200/csrc/htile_gemm.cu,
int8_tc_kernel) relies on for bit-exact outputs, checked exhaustively on the host.

1. Plug nibbles to int8: for a byte n in 0..15, ((n + 0x78) ^ 0x80) is n - 8 as int8, and
   the add never carries into the next byte, so four nibbles per 32-bit word convert at
   once (unpack32).
2. Block sums to float: a 64-k block of int8 products sums to |s| <= 64 * 128 * 128 =
   2^20; the bits 0x4B400000 + s read as an f32, minus 1.5 * 2^23, equal (float)s exactly
   (the epilogue's replacement for the int-to-float conversion).
"""
import numpy as np


def test_nibble_to_int8_per_byte():
    n = np.arange(16, dtype=np.uint32)
    got = ((n + 0x78) ^ 0x80) & 0xFF
    want = (n.astype(np.int32) - 8).astype(np.int8).view(np.uint8).astype(np.uint32)
    assert np.array_equal(got, want)


def test_nibble_to_int8_four_bytes_no_carry():
    # every combination of the extreme nibbles in the four byte lanes, plus random words
    rng = np.random.default_rng(0)
    ext = np.array([0, 7, 8, 15], dtype=np.uint32)
    lanes = np.stack(np.meshgrid(ext, ext, ext, ext, indexing="ij"), -1).reshape(-1, 4)
    lanes = np.concatenate([lanes, rng.integers(0, 16, (4096, 4), dtype=np.uint32)])
    words = lanes[:, 0] | (lanes[:, 1] << 8) | (lanes[:, 2] << 16) | (lanes[:, 3] << 24)
    out = ((words + np.uint32(0x78787878)) ^ np.uint32(0x80808080)).astype(np.uint32)
    got = out.view(np.uint8).reshape(-1, 4).view(np.int8)
    assert np.array_equal(got, lanes.astype(np.int32) - 8)


def test_biased_int32_reads_as_exact_float():
    s = np.arange(-(1 << 20), (1 << 20) + 1, dtype=np.int64)
    bits = (s + 0x4B400000).astype(np.uint32)
    f = bits.view(np.float32) - np.float32(12582912.0)
    assert f.dtype == np.float32
    assert np.array_equal(f, s.astype(np.float32))
