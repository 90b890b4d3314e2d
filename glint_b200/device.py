"""libglint_encode.so on torch CUDA tensors: device pointers, stream ordered.

Every call goes through the library's C ABI (the same entry points a C or ctypes
caller binds); torch only owns the memory and the stream.  There is no CPU
fallback: a missing library or a non-CUDA tensor raises.
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence, Tuple

import torch

from . import glint_cuda

PRECISE, FAST = 0, 1
_MODES = {"precise": PRECISE, "fast": FAST, PRECISE: PRECISE, FAST: FAST}


class GlintTensorDesc(ctypes.Structure):
    """struct GlintTensorDesc of include/glint_encode.h."""
    _fields_ = [
        ("dense", ctypes.c_void_p),
        ("hole_packed", ctypes.c_void_p),
        ("plug_packed", ctypes.c_void_p),
        ("absmax", ctypes.c_void_p),
        ("n", ctypes.c_int64),
    ]


def lib():
    L = glint_cuda.load()
    if L is None:
        raise RuntimeError(glint_cuda._ERR or "libglint_encode.so not loaded")
    return L


def _stream(stream: Optional[torch.cuda.Stream] = None) -> ctypes.c_void_p:
    s = stream if stream is not None else torch.cuda.current_stream()
    return ctypes.c_void_p(s.cuda_stream)


def _check(rc: int, what: str) -> None:
    if rc != 0:
        raise RuntimeError(f"{what} rc={rc}")


def _cuda(t: torch.Tensor, name: str) -> None:
    if not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor")
    if not t.is_contiguous():
        raise ValueError(f"{name} must be contiguous")


def n_packed(n: int) -> int:
    return (n + 1) // 2


def n_absmax(n: int, blocksize: int) -> int:
    return (n + blocksize - 1) // blocksize if blocksize > 0 and n > 0 else 0


def alloc_planes(n: int, blocksize: int, device) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    return (torch.empty(n_packed(n), dtype=torch.uint8, device=device),
            torch.empty(n_packed(n), dtype=torch.uint8, device=device),
            torch.empty(n_absmax(n, blocksize), dtype=torch.float32, device=device))


def encode(w: torch.Tensor, blocksize: int = 64, out=None, stream=None):
    """BF16 or f32 CUDA tensor (any shape, flattened) -> (hole u8, plug u8, absmax f32)."""
    _cuda(w, "w")
    n = w.numel()
    hole, plug, am = out if out is not None else alloc_planes(n, blocksize, w.device)
    if w.dtype == torch.bfloat16:
        fn, name = lib().glint_encode_bf16_device, "glint_encode_bf16_device"
    elif w.dtype == torch.float32:
        fn, name = lib().glint_encode_f32_device, "glint_encode_f32_device"
    else:
        raise ValueError(f"encode takes bfloat16 or float32, not {w.dtype}")
    _check(fn(w.data_ptr(), n, blocksize, hole.data_ptr(), plug.data_ptr(), am.data_ptr(), _stream(stream)), name)
    return hole, plug, am


def _descs(items: Sequence[Tuple[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor]]):
    arr = (GlintTensorDesc * max(1, len(items)))()
    for i, (dense, h, p, a) in enumerate(items):
        arr[i] = GlintTensorDesc(dense.data_ptr(), h.data_ptr(), p.data_ptr(), a.data_ptr(), dense.numel())
    return arr


def encode_batch(ws: Sequence[torch.Tensor], blocksize: int = 64, outs=None, stream=None) -> List[tuple]:
    """Encode many BF16 tensors with few launches."""
    for w in ws:
        _cuda(w, "w")
        if w.dtype != torch.bfloat16:
            raise ValueError("encode_batch takes bfloat16 tensors")
    outs = outs if outs is not None else [alloc_planes(w.numel(), blocksize, w.device) for w in ws]
    arr = _descs([(w, *o) for w, o in zip(ws, outs)])
    _check(lib().glint_encode_bf16_device_batch(arr, len(ws), blocksize, _stream(stream)),
           "glint_encode_bf16_device_batch")
    return list(outs)


def expand(hole: torch.Tensor, plug: torch.Tensor, absmax: torch.Tensor, n: int, blocksize: int = 64,
           dtype: torch.dtype = torch.bfloat16, out=None, stream=None) -> torch.Tensor:
    """Packed planes -> n dense weights (BF16 or f32)."""
    for t, nm in ((hole, "hole"), (plug, "plug"), (absmax, "absmax")):
        _cuda(t, nm)
    out = out if out is not None else torch.empty(n, dtype=dtype, device=hole.device)
    if out.dtype == torch.bfloat16:
        fn, name = lib().glint_expand_packed_to_bf16_device, "glint_expand_packed_to_bf16_device"
    elif out.dtype == torch.float32:
        fn, name = lib().glint_expand_packed_to_f32_device, "glint_expand_packed_to_f32_device"
    else:
        raise ValueError(f"expand writes bfloat16 or float32, not {out.dtype}")
    _check(fn(hole.data_ptr(), plug.data_ptr(), absmax.data_ptr(), n, blocksize, out.data_ptr(), _stream(stream)),
           name)
    return out


def expand_batch(planes: Sequence[tuple], outs: Sequence[torch.Tensor], blocksize: int = 64, stream=None):
    """planes[i] = (hole, plug, absmax); outs[i] BF16 tensors of the dense sizes."""
    arr = _descs([(o, *pl) for o, pl in zip(outs, planes)])
    _check(lib().glint_expand_packed_to_bf16_device_batch(arr, len(outs), blocksize, _stream(stream)),
           "glint_expand_packed_to_bf16_device_batch")
    return outs


def htile(x: torch.Tensor, hole: torch.Tensor, plug: torch.Tensor, absmax: torch.Tensor, N: int,
          blocksize: int = 64, mode="precise", out_dtype: torch.dtype = torch.float32, out=None,
          stream=None) -> torch.Tensor:
    """y[M, N] = x[M, K] @ W^T, W given as GLINT planes of the [N, K] weight."""
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.dim() != 2:
        raise ValueError("x must be a 2-D bfloat16 tensor [M, K]")
    M, K = x.shape
    out = out if out is not None else torch.empty((M, N), dtype=out_dtype, device=x.device)
    ydt = 1 if out.dtype == torch.bfloat16 else 0
    if out.dtype not in (torch.bfloat16, torch.float32):
        raise ValueError("y must be float32 or bfloat16")
    rc = lib().glint_htile_stream(hole.data_ptr(), plug.data_ptr(), absmax.data_ptr(), x.data_ptr(), out.data_ptr(),
                                  ydt, M, N, K, blocksize, _MODES[mode], _stream(stream))
    _check(rc, "glint_htile_stream")
    return out


def htile_reference_abi(x: torch.Tensor, hole, plug, absmax, N: int, blocksize: int = 64, out=None,
                        stream=None) -> torch.Tensor:
    """The reference's own entry point launch_glint_htile_s3_f32_stream (f32 y)."""
    M, K = x.shape
    out = out if out is not None else torch.empty((M, N), dtype=torch.float32, device=x.device)
    rc = lib().launch_glint_htile_s3_f32_stream(hole.data_ptr(), plug.data_ptr(), absmax.data_ptr(), x.data_ptr(),
                                                out.data_ptr(), M, N, K, blocksize, _stream(stream))
    _check(rc, "launch_glint_htile_s3_f32_stream")
    return out


# ---- K-major decode: parent-only GEMV + activation-selected plug correction ----
# (include/glint_km.h; the reference's Mojo decoders' glint_gemv_km, select_topk,
# apply_corr_k, transpose_plug / transpose_scales)

def to_kmajor(hole: torch.Tensor, plug: torch.Tensor, absmax: torch.Tensor, N: int, K: int, blocksize: int = 64,
              plug_out: Optional[torch.Tensor] = None, stream=None):
    """(hole_k, plug_k, scales_k) of a GLINT weight [N, K]: planes [K, N/2] bytes
    (row r of channel c in nibble r & 1 of byte c*N/2 + r/2), scales [K/64, N] f32.
    plug_out may be a pinned host tensor to receive plug_k (copied after the
    device transform), for a decode that reads plug rows from host memory."""
    for t, nm in ((hole, "hole"), (plug, "plug"), (absmax, "absmax")):
        _cuda(t, nm)
    dev = hole.device
    hk = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
    pk = torch.empty(K * N // 2, dtype=torch.uint8, device=dev)
    sk = torch.empty((K // 64) * N, dtype=torch.float32, device=dev)
    rc = lib().glint_kmajor_from_rowmajor(hole.data_ptr(), plug.data_ptr(), absmax.data_ptr(), N, K, blocksize,
                                          hk.data_ptr(), pk.data_ptr(), sk.data_ptr(), _stream(stream))
    _check(rc, "glint_kmajor_from_rowmajor")
    if plug_out is not None:
        plug_out.copy_(pk, non_blocking=True)
        pk = plug_out
    return hk, pk, sk


def _x_vec(x: torch.Tensor) -> torch.Tensor:
    _cuda(x, "x")
    if x.dtype != torch.bfloat16 or x.numel() != x.shape[-1] or x.dim() > 2:
        raise ValueError("x must be one bfloat16 row [K] or [1, K]")
    return x


def _plug_ptr(plug_k: torch.Tensor) -> int:
    if not (plug_k.is_cuda or plug_k.is_pinned()):
        raise ValueError("plug_k must be a CUDA tensor or pinned host memory")
    if not plug_k.is_contiguous():
        raise ValueError("plug_k must be contiguous")
    return plug_k.data_ptr()


def gemv_km(x: torch.Tensor, hole_k: torch.Tensor, scales_k: torch.Tensor, N: int, out=None,
            stream=None) -> torch.Tensor:
    """Parent-only y[N] = sum_c PARENT[h] * scale * x[c] (M = 1), f32."""
    x = _x_vec(x)
    K = x.shape[-1]
    y = out if out is not None else torch.empty(N, dtype=torch.float32, device=x.device)
    rc = lib().glint_gemv_km_stream(hole_k.data_ptr(), scales_k.data_ptr(), x.data_ptr(), y.data_ptr(), N, K,
                                    _stream(stream))
    _check(rc, "glint_gemv_km_stream")
    return y


def select_topk(x: torch.Tensor, nsel: int, idx=None, cnt=None, stream=None):
    """(idx [K] int32, cnt [1] int32): the channels kept by the |x| rule, ascending
    in idx[:cnt]; both stay on the device."""
    x = _x_vec(x)
    K = x.shape[-1]
    idx = idx if idx is not None else torch.empty(K, dtype=torch.int32, device=x.device)
    cnt = cnt if cnt is not None else torch.empty(1, dtype=torch.int32, device=x.device)
    rc = lib().glint_select_topk_stream(x.data_ptr(), K, nsel, idx.data_ptr(), cnt.data_ptr(), _stream(stream))
    _check(rc, "glint_select_topk_stream")
    return idx, cnt


def apply_corr_k(y: torch.Tensor, x: torch.Tensor, hole_k, plug_k, scales_k, idx, cnt, N: int,
                 stream=None) -> torch.Tensor:
    """y += sum over the selected channels of (CELLS - PARENT)[h][p] * scale * x[c], in place."""
    x = _x_vec(x)
    K = x.shape[-1]
    rc = lib().glint_apply_corr_k_stream(hole_k.data_ptr(), _plug_ptr(plug_k), scales_k.data_ptr(), x.data_ptr(),
                                         idx.data_ptr(), cnt.data_ptr(), y.data_ptr(), N, K, _stream(stream))
    _check(rc, "glint_apply_corr_k_stream")
    return y


def gemv_select(x: torch.Tensor, hole_k, plug_k, scales_k, N: int, nsel: int, out=None, idx=None, cnt=None,
                stream=None):
    """One decode step: select the channels, parent GEMV, plug correction.
    Returns (y [N] f32, idx, cnt)."""
    x = _x_vec(x)
    K = x.shape[-1]
    y = out if out is not None else torch.empty(N, dtype=torch.float32, device=x.device)
    idx = idx if idx is not None else torch.empty(K, dtype=torch.int32, device=x.device)
    cnt = cnt if cnt is not None else torch.empty(1, dtype=torch.int32, device=x.device)
    rc = lib().glint_gemv_select_stream(hole_k.data_ptr(), _plug_ptr(plug_k), scales_k.data_ptr(), x.data_ptr(),
                                        y.data_ptr(), N, K, nsel, idx.data_ptr(), cnt.data_ptr(), _stream(stream))
    _check(rc, "glint_gemv_select_stream")
    return y, idx, cnt
