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
