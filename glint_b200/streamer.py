"""Python handle for the plug streamer C ABI (include/glint_plug_streamer.h).

The reference drives its streamer from C (cuda/glint_plug_streamer.cu:27-215,
tests/test_glint_plug_streamer.cu); this wrapper exposes the same calls with the
same return codes for Python callers and tests.  Streams are passed as raw
cudaStream_t handles (e.g. `torch.cuda.Stream().cuda_stream`).
"""
from __future__ import annotations

import ctypes
from typing import Sequence, Tuple

from . import glint_cuda


class _DeviceBytes:
    """A device byte range as a CUDA array (for torch.as_tensor), no copy."""

    def __init__(self, ptr: int, nbytes: int):
        self.__cuda_array_interface__ = {"shape": (nbytes,), "typestr": "|u1", "data": (ptr, False),
                                         "version": 2}


def device_bytes(ptr: int, nbytes: int):
    """torch uint8 view of `nbytes` device bytes at `ptr` (no copy, no ownership)."""
    import torch
    return torch.as_tensor(_DeviceBytes(ptr, nbytes), device="cuda")


class PlugStreamer:
    """Two-slot VRAM ring for per-layer plug planes held in pinned host memory."""

    def __init__(self, layer_bytes: Sequence[int], copy_stream: int, compute_stream: int):
        self._lib = glint_cuda._require()
        self.layer_bytes = [int(b) for b in layer_bytes]
        arr = (ctypes.c_uint64 * len(self.layer_bytes))(*self.layer_bytes)
        h = ctypes.c_void_p()
        rc = self._lib.glint_plug_streamer_create(ctypes.byref(h), len(self.layer_bytes), arr,
                                                  ctypes.c_void_p(copy_stream), ctypes.c_void_p(compute_stream))
        if rc != 0:
            raise RuntimeError(f"glint_plug_streamer_create rc={rc}")
        self._h = h

    @property
    def n_layers(self) -> int:
        return len(self.layer_bytes)

    def set_host_data(self, layer: int, data) -> int:
        """Copy a layer's plug bytes (bytes, numpy array or CPU tensor) into pinned memory."""
        if hasattr(data, "data_ptr"):
            ptr, n = data.data_ptr(), data.numel() * data.element_size()
        elif hasattr(data, "ctypes"):
            ptr, n = data.ctypes.data, data.nbytes
        else:
            buf = ctypes.create_string_buffer(bytes(data), len(data))
            ptr, n = ctypes.addressof(buf), len(data)
        return self._lib.glint_plug_streamer_set_host_data(self._h, layer, ctypes.c_void_p(ptr), n)

    def host_buffer(self, layer: int):
        """numpy uint8 view of the layer's pinned host buffer (write plugs in place)."""
        import numpy as np
        p = self._lib.glint_plug_streamer_host_buffer(self._h, layer)
        if not p:
            raise IndexError(layer)
        return np.ctypeslib.as_array((ctypes.c_uint8 * self.layer_bytes[layer]).from_address(p))

    def start(self) -> int:
        return self._lib.glint_plug_streamer_start(self._h)

    def acquire(self, layer: int) -> Tuple[int, int]:
        """(rc, device pointer of the layer's slot)."""
        p = ctypes.c_void_p()
        rc = self._lib.glint_plug_streamer_acquire(self._h, layer, ctypes.byref(p))
        return rc, (p.value or 0)

    def release(self, layer: int) -> int:
        return self._lib.glint_plug_streamer_release(self._h, layer)

    def stats(self) -> dict:
        st = glint_cuda.StreamerStats()
        rc = self._lib.glint_plug_streamer_get_stats(self._h, ctypes.byref(st))
        if rc != 0:
            raise RuntimeError(f"glint_plug_streamer_get_stats rc={rc}")
        return {"total_h2d_bytes": st.total_h2d_bytes, "total_stall_ms": st.total_stall_ms,
                "per_layer_stall_ms": list(st.per_layer_stall_ms[: st.n_layers]), "n_layers": st.n_layers}

    def reset_stats(self) -> None:
        self._lib.glint_plug_streamer_reset_stats(self._h)

    def close(self) -> None:
        if self._h:
            self._lib.glint_plug_streamer_destroy(self._h)
            self._h = None

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
