"""ctypes front end of libglint_encode.so with the reference's interface.

Mirrors Jadon-Fox/glint glint_cuda.py:1-85 name for name (lib_path, load,
encode_bf16_cuda, expand_cuda, gpu_ok) with the same argument meaning, return
values and errors (RuntimeError carrying rc=...), so the reference's
glint_pin.py (`from glint_cuda import encode_bf16_cuda, load`) and
glint_verify.py (`from glint_cuda import expand_cuda`) run on this library
unchanged.  Lookup order as the reference: $GLINT_ENCODE_SO, then the in-tree
build.  Added: expand_bf16_cuda (the BF16 bytes glint_unpin.py writes) and
encode_f32_cuda.
"""
from __future__ import annotations

import ctypes
import os
from pathlib import Path
from typing import Optional, Tuple

from .build import PKG, LIB_NAME

_LIB = None
_ERR = None


def lib_path() -> Optional[Path]:
    env = os.environ.get("GLINT_ENCODE_SO")
    if env:
        p = Path(env)
        return p if p.is_file() else None
    p = PKG / LIB_NAME
    return p if p.is_file() else None


def _bind(lib):
    vp, i64, i32 = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.glint_encode_n_absmax.argtypes = [i64, i32]
    lib.glint_encode_n_absmax.restype = i32
    lib.glint_encode_n_packed.argtypes = [i64]
    lib.glint_encode_n_packed.restype = i32
    lib.glint_encode_n_absmax64.argtypes = [i64, i32]
    lib.glint_encode_n_absmax64.restype = i64
    lib.glint_encode_n_packed64.argtypes = [i64]
    lib.glint_encode_n_packed64.restype = i64
    for f in (lib.glint_encode_bf16_host, lib.glint_encode_f32_host):
        f.argtypes = [vp, i64, i32, vp, vp, vp]
        f.restype = i32
    for f in (lib.glint_expand_packed_to_f32_host, lib.glint_expand_packed_to_bf16_host):
        f.argtypes = [vp, vp, vp, i64, i32, vp]
        f.restype = i32
    for f in (lib.glint_encode_bf16_host_sqerr, lib.glint_encode_f32_host_sqerr):
        f.argtypes = [vp, i64, i32, vp, vp, vp, ctypes.POINTER(ctypes.c_double)]
        f.restype = i32
    lib.glint_cells_f32.argtypes = [vp]
    lib.glint_cells_f32.restype = i32
    for f in (lib.glint_encode_bf16_device, lib.glint_encode_f32_device):
        f.argtypes = [vp, i64, i32, vp, vp, vp, vp]
        f.restype = i32
    for f in (lib.glint_expand_packed_to_f32_device, lib.glint_expand_packed_to_bf16_device):
        f.argtypes = [vp, vp, vp, i64, i32, vp, vp]
        f.restype = i32
    for f in (lib.glint_encode_bf16_device_batch, lib.glint_expand_packed_to_bf16_device_batch):
        f.argtypes = [vp, i32, i32, vp]
        f.restype = i32
    for f in (lib.launch_glint_htile_s3_f32_stream,):
        f.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, vp]
        f.restype = i32
    lib.launch_glint_htile_s3_f32.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32]
    lib.launch_glint_htile_s3_f32.restype = i32
    lib.glint_htile_stream.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]
    lib.glint_htile_stream.restype = i32
    lib.p7_abi_version.restype = ctypes.c_char_p
    lib.glint_b200_version.restype = ctypes.c_char_p
    # gathered decode and CUDA IPC (include/glint_htile.h, additive)
    lib.glint_htile_gather_stream.argtypes = [vp, vp, vp, vp, ctypes.POINTER(vp), ctypes.POINTER(vp), i32, i32, i32,
                                              i32, i32, i32, i32, i32, i32, i32, vp]
    lib.glint_htile_gather_stream.restype = i32
    lib.glint_gather_stream.argtypes = [vp, i32, i32, i32, i32, ctypes.POINTER(vp), ctypes.POINTER(vp), i32, i32,
                                        i32, i32, vp]
    lib.glint_gather_stream.restype = i32
    lib.glint_device_alloc.argtypes = [ctypes.c_size_t, ctypes.POINTER(vp)]
    lib.glint_device_alloc.restype = i32
    lib.glint_device_free.argtypes = [vp]
    lib.glint_device_free.restype = i32
    lib.glint_ipc_handle.argtypes = [vp, vp]
    lib.glint_ipc_handle.restype = i32
    lib.glint_ipc_open.argtypes = [vp, ctypes.POINTER(vp)]
    lib.glint_ipc_open.restype = i32
    lib.glint_ipc_close.argtypes = [vp]
    lib.glint_ipc_close.restype = i32
    # K-major decode (include/glint_km.h, additive)
    lib.glint_kmajor_from_rowmajor.argtypes = [vp, vp, vp, i32, i32, i32, vp, vp, vp, vp]
    lib.glint_gemv_km_stream.argtypes = [vp, vp, vp, vp, i32, i32, vp]
    lib.glint_select_topk_stream.argtypes = [vp, i32, i32, vp, vp, vp]
    lib.glint_apply_corr_k_stream.argtypes = [vp, vp, vp, vp, vp, vp, vp, i32, i32, vp]
    lib.glint_gemv_select_stream.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, vp, vp, vp]
    for f in (lib.glint_kmajor_from_rowmajor, lib.glint_gemv_km_stream, lib.glint_select_topk_stream,
              lib.glint_apply_corr_k_stream, lib.glint_gemv_select_stream):
        f.restype = i32
    # plug streamer (include/glint_plug_streamer.h)
    lib.glint_plug_streamer_create.argtypes = [ctypes.POINTER(vp), i32, ctypes.POINTER(ctypes.c_uint64), vp, vp]
    lib.glint_plug_streamer_create.restype = i32
    lib.glint_plug_streamer_destroy.argtypes = [vp]
    lib.glint_plug_streamer_destroy.restype = None
    lib.glint_plug_streamer_set_host_data.argtypes = [vp, i32, vp, ctypes.c_uint64]
    lib.glint_plug_streamer_set_host_data.restype = i32
    lib.glint_plug_streamer_start.argtypes = [vp]
    lib.glint_plug_streamer_start.restype = i32
    lib.glint_plug_streamer_acquire.argtypes = [vp, i32, ctypes.POINTER(vp)]
    lib.glint_plug_streamer_acquire.restype = i32
    lib.glint_plug_streamer_release.argtypes = [vp, i32]
    lib.glint_plug_streamer_release.restype = i32
    lib.glint_plug_streamer_get_stats.argtypes = [vp, ctypes.POINTER(StreamerStats)]
    lib.glint_plug_streamer_get_stats.restype = i32
    lib.glint_plug_streamer_reset_stats.argtypes = [vp]
    lib.glint_plug_streamer_reset_stats.restype = None
    lib.glint_plug_streamer_host_buffer.argtypes = [vp, i32]
    lib.glint_plug_streamer_host_buffer.restype = vp
    return lib


class StreamerStats(ctypes.Structure):
    """GlintStreamerStats (include/glint_plug_streamer.h)."""
    _fields_ = [("total_h2d_bytes", ctypes.c_uint64), ("total_stall_ms", ctypes.c_double),
                ("per_layer_stall_ms", ctypes.c_double * 64), ("n_layers", ctypes.c_int)]


def load():
    """The loaded library, or None with the reason kept for encode_bf16_cuda's error."""
    global _LIB, _ERR
    if _LIB is not None:
        return _LIB
    p = lib_path()
    if p is None:
        _ERR = "libglint_encode.so not found - build it with `make -C glint_b200/csrc` (nvcc, sm_100a)"
        return None
    _LIB = _bind(ctypes.CDLL(str(p)))
    return _LIB


def _require():
    lib = load()
    if lib is None:
        raise RuntimeError(_ERR)
    return lib


def encode_bf16_cuda(raw_bf16: bytes, n: int, blocksize: int = 64) -> Tuple[bytes, bytes, bytes]:
    """BF16 bytes (n weights) -> (hole bytes, plug bytes, absmax f32 bytes)."""
    lib = _require()
    n_am = lib.glint_encode_n_absmax(n, blocksize)
    n_pk = lib.glint_encode_n_packed(n)
    hole = (ctypes.c_uint8 * n_pk)()
    plug = (ctypes.c_uint8 * n_pk)()
    am = (ctypes.c_float * n_am)()
    buf = (ctypes.c_uint16 * n).from_buffer_copy(raw_bf16[: n * 2])
    rc = lib.glint_encode_bf16_host(ctypes.addressof(buf), n, blocksize, ctypes.addressof(hole),
                                    ctypes.addressof(plug), ctypes.addressof(am))
    if rc != 0:
        raise RuntimeError(f"glint_encode_bf16_host rc={rc}")
    return bytes(hole), bytes(plug), bytes(ctypes.string_at(ctypes.addressof(am), n_am * 4))


def encode_f32_cuda(raw_f32: bytes, n: int, blocksize: int = 64) -> Tuple[bytes, bytes, bytes]:
    lib = _require()
    n_am = lib.glint_encode_n_absmax(n, blocksize)
    n_pk = lib.glint_encode_n_packed(n)
    hole = (ctypes.c_uint8 * n_pk)()
    plug = (ctypes.c_uint8 * n_pk)()
    am = (ctypes.c_float * n_am)()
    buf = (ctypes.c_float * n).from_buffer_copy(raw_f32[: n * 4])
    rc = lib.glint_encode_f32_host(ctypes.addressof(buf), n, blocksize, ctypes.addressof(hole),
                                   ctypes.addressof(plug), ctypes.addressof(am))
    if rc != 0:
        raise RuntimeError(f"glint_encode_f32_host rc={rc}")
    return bytes(hole), bytes(plug), bytes(ctypes.string_at(ctypes.addressof(am), n_am * 4))


def expand_cuda(hole: bytes, plug: bytes, absmax_f32: bytes, n: int, blocksize: int = 64) -> bytes:
    """GPU expand -> n little-endian f32 (reference glint_cuda.expand_cuda)."""
    lib = _require()
    out = (ctypes.c_float * n)()
    h = ctypes.create_string_buffer(bytes(hole), len(hole))
    p = ctypes.create_string_buffer(bytes(plug), len(plug))
    a = ctypes.create_string_buffer(bytes(absmax_f32), len(absmax_f32))
    rc = lib.glint_expand_packed_to_f32_host(h, p, a, n, blocksize, ctypes.addressof(out))
    if rc != 0:
        raise RuntimeError(f"glint_expand_packed_to_f32_host rc={rc}")
    return bytes(ctypes.string_at(ctypes.addressof(out), n * 4))


def expand_bf16_cuda(hole: bytes, plug: bytes, absmax_f32: bytes, n: int, blocksize: int = 64) -> bytes:
    """GPU expand -> n little-endian BF16, the bytes glint_unpin.py writes for BF16."""
    lib = _require()
    out = (ctypes.c_uint16 * n)()
    h = ctypes.create_string_buffer(bytes(hole), len(hole))
    p = ctypes.create_string_buffer(bytes(plug), len(plug))
    a = ctypes.create_string_buffer(bytes(absmax_f32), len(absmax_f32))
    rc = lib.glint_expand_packed_to_bf16_host(h, p, a, n, blocksize, ctypes.addressof(out))
    if rc != 0:
        raise RuntimeError(f"glint_expand_packed_to_bf16_host rc={rc}")
    return bytes(ctypes.string_at(ctypes.addressof(out), n * 2))


def gpu_ok() -> bool:
    """Library loads and a 2-weight encode runs. False on a box with no GPU."""
    try:
        encode_bf16_cuda(b"\x80\x3f\x00\x00", 2, 64)
        return True
    except (RuntimeError, OSError):
        return False


def require_gpu(work: str = "GLINT encode", host_path: str = "the reference's glint_pin.py --allow-cpu"):
    """The loaded library when a GPU can run it; RuntimeError otherwise, naming `work`
    and the reference tool that is the host path (the front ends here have none)."""
    lib = load()
    if lib is None:
        raise RuntimeError(f"{work} is CUDA (libglint_encode.so): {_ERR}")
    if not gpu_ok():
        raise RuntimeError(f"{work} is CUDA: libglint_encode.so loaded but no usable GPU; there is no host "
                           f"path here ({host_path} is one)")
    return lib
