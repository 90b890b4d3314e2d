"""INT8 W8A8 GEMM with the res4 late plug on torch CUDA tensors, through the C ABI of
include/int8_mma_gemm.h (the reference's cuda/int8_mma_gemm.cu entry points, exported
by libglint_encode.so).  `lib` may be any library exporting that ABI; by default this
repository's.  No CPU fallback: non-CUDA tensors or a missing library raise."""
from __future__ import annotations

import ctypes
from typing import Optional, Tuple

import torch


class Int8MmaLinear(ctypes.Structure):
    """struct Int8MmaLinear of include/int8_mma_gemm.h (passed by value)."""
    _fields_ = [("q", ctypes.c_void_p), ("scale", ctypes.c_void_p), ("n_out", ctypes.c_int), ("k_in", ctypes.c_int)]


def bind(lib: ctypes.CDLL) -> ctypes.CDLL:
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    lib.int8_mma_gemm.argtypes = [vp, Int8MmaLinear, vp, i32, vp, vp, vp]
    lib.int8_mma_gemm_plug.argtypes = [vp, Int8MmaLinear, vp, vp, vp, i32, vp, vp, vp, vp]
    lib.int8_mma_gemm_plug_fused.argtypes = [vp, Int8MmaLinear, vp, vp, vp, i32, vp, vp, vp]
    lib.int8_mma_gemm_resolve.argtypes = [vp, Int8MmaLinear, vp, vp, vp, i32, vp, vp, vp, vp, vp, vp]
    for f in (lib.int8_mma_gemm, lib.int8_mma_gemm_plug, lib.int8_mma_gemm_plug_fused, lib.int8_mma_gemm_resolve):
        f.restype = ctypes.c_int  # cudaError_t
    return lib


def _ours() -> ctypes.CDLL:
    from . import glint_cuda
    lib = glint_cuda.load()
    if lib is None:
        raise RuntimeError(glint_cuda._ERR or "libglint_encode.so not loaded")
    if not getattr(lib, "_int8_bound", False):
        bind(lib)
        lib._int8_bound = True
    return lib


def _p(t: Optional[torch.Tensor]):
    return None if t is None else t.data_ptr()


def gemm(x: torch.Tensor, q: torch.Tensor, scale: torch.Tensor, plug: Optional[Tuple[torch.Tensor, torch.Tensor]] = None,
         kind: str = "gemm", out: Optional[torch.Tensor] = None, scratch=None, lib: Optional[ctypes.CDLL] = None,
         stream=None):
    """y [m, n_out] f32 = x [m, k_in] (BF16) . (q * scale [+ plug])^T.

    kind: "gemm" (no plug), "plug" (two passes, plug_i8 scratch), "fused" (one pass) or
    "resolve" (with the activation's quantization residual; plug optional).  Returns
    (y, scratch) where scratch holds the quantized activations (xq, sx[, rq, sr]) and
    the unpacked plug, as the C calls fill them."""
    lib = lib or _ours()
    m, k = x.shape
    n = q.shape[0]
    dev = x.device
    y = out if out is not None else torch.empty((m, n), dtype=torch.float32, device=dev)
    sc = scratch or {}
    sc.setdefault("xq", torch.empty(m * k, dtype=torch.int8, device=dev))
    sc.setdefault("sx", torch.empty(m * (k // 64), dtype=torch.float32, device=dev))
    lin = Int8MmaLinear(q.data_ptr(), scale.data_ptr(), n, k)
    s = ctypes.c_void_p((stream if stream is not None else torch.cuda.current_stream()).cuda_stream)
    pq, ps = (plug if plug is not None else (None, None))
    if kind == "gemm":
        rc = lib.int8_mma_gemm(x.data_ptr(), lin, y.data_ptr(), m, _p(sc["xq"]), _p(sc["sx"]), s)
    elif kind == "plug":
        sc.setdefault("plug_i8", torch.empty(n * k, dtype=torch.int8, device=dev))
        rc = lib.int8_mma_gemm_plug(x.data_ptr(), lin, _p(pq), _p(ps), y.data_ptr(), m, _p(sc["xq"]), _p(sc["sx"]),
                                    _p(sc["plug_i8"]), s)
    elif kind == "fused":
        rc = lib.int8_mma_gemm_plug_fused(x.data_ptr(), lin, _p(pq), _p(ps), y.data_ptr(), m, _p(sc["xq"]),
                                          _p(sc["sx"]), s)
    elif kind == "resolve":
        sc.setdefault("rq", torch.empty(m * k, dtype=torch.int8, device=dev))
        sc.setdefault("sr", torch.empty(m * (k // 64), dtype=torch.float32, device=dev))
        if plug is not None:
            sc.setdefault("plug_i8", torch.empty(n * k, dtype=torch.int8, device=dev))
        rc = lib.int8_mma_gemm_resolve(x.data_ptr(), lin, _p(pq), _p(ps), y.data_ptr(), m, _p(sc["xq"]),
                                       _p(sc["sx"]), _p(sc["rq"]), _p(sc["sr"]),
                                       _p(sc.get("plug_i8")) if plug is not None else None, s)
    else:
        raise ValueError(f"unknown kind {kind}")
    if rc != 0:
        raise RuntimeError(f"int8_mma_gemm ({kind}) returned cudaError {rc}")
    return y, sc
