"""GLINT CPU oracle loader — TEST INFRASTRUCTURE ONLY.

numpy front end over oracle/libglint_oracle.so (oracle/glint_oracle.c), the C
restatement of the reference's kernel-exact codec (glint_np.py, glint_encode.cu,
glint_htile.cu of Jadon-Fox/glint).  Only tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline leg import this module; the product never does.

Also locates the reference's own CUDA libraries built for sm_100a under
oracle/_ref/ (see oracle/Makefile), used by GPU tests as a second checker.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
_LIB = None


def reference_checkout() -> Path | None:
    """The read-only reference checkout: GLINT_REFERENCE if set, else a checkout named
    `reference` beside this repository; None when neither exists."""
    env = os.environ.get("GLINT_REFERENCE")
    cand = Path(env) if env else HERE.parent.parent / "reference"
    return cand if (cand / "cuda" / "glint_encode.cu").is_file() else None


def build() -> Path:
    """Compile the oracle (and oracle/_ref when the reference checkout is present)."""
    env = dict(os.environ)
    ref = reference_checkout()
    if ref is not None:
        env["GLINT_REFERENCE"] = str(ref)
    subprocess.run(["make", "-s", "-C", str(HERE)], check=True, env=env)
    return HERE / "libglint_oracle.so"


def lib():
    global _LIB
    if _LIB is not None:
        return _LIB
    p = HERE / "libglint_oracle.so"
    if not p.is_file():
        build()
    L = ctypes.CDLL(str(p))
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    L.orc_set_threads.argtypes = [i32]
    L.orc_max_threads.restype = i32
    L.orc_code.argtypes = [ctypes.c_float]
    L.orc_code.restype = i32
    L.orc_codes_for_bits.argtypes = [ctypes.c_uint32, i64, vp]
    for f in (L.orc_encode_f32, L.orc_encode_bf16):
        f.argtypes = [vp, i64, i32, vp, vp, vp]
        f.restype = i32
    for f in (L.orc_expand_f32, L.orc_expand_bf16):
        f.argtypes = [vp, vp, vp, i64, i32, vp]
        f.restype = i32
    L.orc_f32_to_bf16.argtypes = [ctypes.c_float]
    L.orc_f32_to_bf16.restype = ctypes.c_uint16
    L.orc_htile.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32]
    L.orc_htile.restype = i32
    L.orc_to_kmajor.argtypes = [vp, vp, vp, i32, i32, vp, vp, vp]
    L.orc_gemv_km.argtypes = [vp, vp, vp, vp, i32, i32, i32]
    L.orc_select_topk.argtypes = [vp, i32, i32, vp]
    L.orc_apply_corr_k.argtypes = [vp, vp, vp, vp, vp, i32, vp, i32, i32]
    for f in (L.orc_to_kmajor, L.orc_gemv_km, L.orc_select_topk, L.orc_apply_corr_k):
        f.restype = i32
    L.orc_int8_quant.argtypes = [vp, vp, vp, i32, i32, vp, vp]
    L.orc_int8_gemm.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp, vp]
    for f in (L.orc_int8_quant, L.orc_int8_gemm):
        f.restype = i32
    _LIB = L
    return L


def set_threads(t: int | None = None) -> int:
    """Use t host threads (default: every core). Returns the count used."""
    L = lib()
    t = t or L.orc_max_threads()
    L.orc_set_threads(t)
    return t


def _ptr(a: np.ndarray) -> int:
    return a.ctypes.data


def encode_bf16(w_bf16: np.ndarray, blocksize: int = 64):
    """BF16 bits (uint16) -> (hole uint8[ceil(n/2)], plug uint8[ceil(n/2)], absmax f32[ceil(n/bs)])."""
    w = np.ascontiguousarray(w_bf16, dtype=np.uint16).reshape(-1)
    n = w.size
    hole = np.zeros((n + 1) // 2, np.uint8)
    plug = np.zeros((n + 1) // 2, np.uint8)
    am = np.zeros((n + blocksize - 1) // blocksize, np.float32)
    rc = lib().orc_encode_bf16(_ptr(w), n, blocksize, _ptr(hole), _ptr(plug), _ptr(am))
    if rc:
        raise ValueError(f"orc_encode_bf16 rc={rc}")
    return hole, plug, am


def encode_f32(w: np.ndarray, blocksize: int = 64):
    w = np.ascontiguousarray(w, dtype=np.float32).reshape(-1)
    n = w.size
    hole = np.zeros((n + 1) // 2, np.uint8)
    plug = np.zeros((n + 1) // 2, np.uint8)
    am = np.zeros((n + blocksize - 1) // blocksize, np.float32)
    rc = lib().orc_encode_f32(_ptr(w), n, blocksize, _ptr(hole), _ptr(plug), _ptr(am))
    if rc:
        raise ValueError(f"orc_encode_f32 rc={rc}")
    return hole, plug, am


def expand_f32(hole, plug, am, n: int, blocksize: int = 64) -> np.ndarray:
    hole = np.ascontiguousarray(hole, np.uint8)
    plug = np.ascontiguousarray(plug, np.uint8)
    am = np.ascontiguousarray(am, np.float32)
    out = np.empty(n, np.float32)
    lib().orc_expand_f32(_ptr(hole), _ptr(plug), _ptr(am), n, blocksize, _ptr(out))
    return out


def expand_bf16(hole, plug, am, n: int, blocksize: int = 64) -> np.ndarray:
    """-> uint16 BF16 bits, RNE with the reference NaN rule."""
    hole = np.ascontiguousarray(hole, np.uint8)
    plug = np.ascontiguousarray(plug, np.uint8)
    am = np.ascontiguousarray(am, np.float32)
    out = np.empty(n, np.uint16)
    lib().orc_expand_bf16(_ptr(hole), _ptr(plug), _ptr(am), n, blocksize, _ptr(out))
    return out


def htile(hole, plug, am, x_bf16: np.ndarray, M: int, N: int, K: int, blocksize: int = 64) -> np.ndarray:
    """y f32 [M,N] = x[M,K] . W^T, W dequantised in f32, summed in f64."""
    hole = np.ascontiguousarray(hole, np.uint8)
    plug = np.ascontiguousarray(plug, np.uint8)
    am = np.ascontiguousarray(am, np.float32)
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    y = np.empty((M, N), np.float32)
    rc = lib().orc_htile(_ptr(hole), _ptr(plug), _ptr(am), _ptr(x), _ptr(y), M, N, K, blocksize)
    if rc:
        raise ValueError(f"orc_htile rc={rc}")
    return y


def to_kmajor(hole, plug, am, n: int, K: int):
    """(hole_k, plug_k, scales_k): planes [K, n/2] bytes (row r of channel c in
    nibble r & 1 of byte c*n/2 + r/2), scales [K/64, n] f32 (transpose_plug /
    transpose_scales of the reference's Mojo decoder)."""
    hole = np.ascontiguousarray(hole, np.uint8)
    plug = np.ascontiguousarray(plug, np.uint8)
    am = np.ascontiguousarray(am, np.float32)
    hk = np.empty(K * n // 2, np.uint8)
    pk = np.empty(K * n // 2, np.uint8)
    sk = np.empty(K // 64 * n, np.float32)
    if lib().orc_to_kmajor(_ptr(hole), _ptr(plug), _ptr(am), n, K, _ptr(hk), _ptr(pk), _ptr(sk)):
        raise ValueError("to_kmajor: n must be even and K a multiple of 64")
    return hk, pk, sk


def gemv_km(hole_k, scales_k, x_bf16: np.ndarray, n: int, K: int, ksg: int = 1) -> np.ndarray:
    """Parent-only y[n] = sum_c PARENT[h] * scale * x[c] (M = 1), the reference's
    f32 order over ksg channel slices."""
    y = np.empty(n, np.float32)
    hk = np.ascontiguousarray(hole_k, np.uint8)
    sk = np.ascontiguousarray(scales_k, np.float32)
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    if lib().orc_gemv_km(_ptr(hk), _ptr(sk), _ptr(x), _ptr(y), n, K, ksg):
        raise ValueError("gemv_km: n % 8 == 0 and K % (64 ksg) == 0 required")
    return y


def select_topk(x_bf16: np.ndarray, nsel: int) -> np.ndarray:
    """Selected input channels (int32, ascending) by the reference's |x| rule."""
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    idx = np.empty(max(1, x.size), np.int32)
    cnt = lib().orc_select_topk(_ptr(x), x.size, nsel, _ptr(idx))
    if cnt < 0:
        raise ValueError("nsel must be >= 0")
    return idx[:cnt].copy()


def apply_corr_k(y: np.ndarray, hole_k, plug_k, scales_k, x_bf16: np.ndarray, idx: np.ndarray, n: int,
                 K: int) -> np.ndarray:
    """y + sum over the selected channels of (CELLS - PARENT)[h][p] * scale * x[c]."""
    out = np.array(y, np.float32, copy=True)
    hk = np.ascontiguousarray(hole_k, np.uint8)
    pk = np.ascontiguousarray(plug_k, np.uint8)
    sk = np.ascontiguousarray(scales_k, np.float32)
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    ix = np.ascontiguousarray(idx, np.int32)
    if lib().orc_apply_corr_k(_ptr(hk), _ptr(pk), _ptr(sk), _ptr(x), _ptr(ix) if ix.size else None, ix.size,
                              _ptr(out), n, K):
        raise ValueError("apply_corr_k: bad arguments")
    return out


def int8_quant(x_bf16: np.ndarray, m: int, k: int, prev=None):
    """(q int8 [m*k], s f32 [m*k/64]) of the activation rule; prev = (q, s) of the
    first pass quantizes its residual (the resolve pass)."""
    x = np.ascontiguousarray(x_bf16, np.uint16).reshape(-1)
    q = np.empty(m * k, np.int8)
    s = np.empty(m * (k // 64), np.float32)
    pq, ps = (None, None) if prev is None else (np.ascontiguousarray(prev[0], np.int8),
                                                np.ascontiguousarray(prev[1], np.float32))
    if lib().orc_int8_quant(_ptr(x), _ptr(pq) if pq is not None else None, _ptr(ps) if ps is not None else None,
                            m, k, _ptr(q), _ptr(s)):
        raise ValueError("int8_quant: k % 64 == 0 and k >= 64 required")
    return q, s


def int8_gemm(xq, sx, wq, sw, m: int, n: int, k: int, y=None, accumulate: bool = False, plug=None) -> np.ndarray:
    """y [m, n] f32 of the INT8 GEMM (plug = (q4 bytes, scales) for the fused late plug)."""
    out = np.zeros((m, n), np.float32) if y is None else np.array(y, np.float32, copy=True)
    args = [np.ascontiguousarray(xq, np.int8), np.ascontiguousarray(sx, np.float32),
            np.ascontiguousarray(wq, np.int8), np.ascontiguousarray(sw, np.float32)]
    pq = ps = None
    if plug is not None:
        pq, ps = np.ascontiguousarray(plug[0], np.uint8), np.ascontiguousarray(plug[1], np.float32)
    if lib().orc_int8_gemm(*[_ptr(a) for a in args], _ptr(out), m, n, k, int(accumulate),
                           _ptr(pq) if pq is not None else None, _ptr(ps) if ps is not None else None):
        raise ValueError("int8_gemm: bad shape")
    return out


def codes_for_bits(lo: int, count: int) -> np.ndarray:
    out = np.empty(count, np.uint8)
    lib().orc_codes_for_bits(lo, count, _ptr(out))
    return out


def f32_to_bf16(a: np.ndarray) -> np.ndarray:
    """RNE f32 -> BF16 bits with the reference NaN rule (glint_np.py:25-31), vectorised."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u + (np.uint32(0x7FFF) + ((u >> 16) & np.uint32(1)))) >> 16).astype(np.uint16)
    return np.where(np.isnan(a), ((u >> 16) | np.uint32(0x40)).astype(np.uint16), r)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, np.uint16).astype(np.uint32) << 16).view(np.float32)


def ref_lib_path(name: str) -> Path | None:
    """oracle/_ref/<name> (the reference's CUDA library built for sm_100a), if built."""
    p = HERE / "_ref" / name
    return p if p.is_file() else None


def cores() -> int:
    return os.cpu_count() or 1
