"""glint_b200: GLINT encode / expand / H-TILE for NVIDIA B200 (sm_100a).

The product is libglint_encode.so (glint_b200/csrc), a C ABI that keeps the
reference's entry points (Jadon-Fox/glint include/glint_encode.h,
include/glint_htile.h, cuda/p7_abi.c).  Python front ends:

  glint_b200.glint_cuda  the reference's glint_cuda.py interface (ctypes, host
                         buffers), so glint_pin.py / glint_verify.py drive it
  glint_b200.device      the same library on torch CUDA tensors (device pointers,
                         stream ordered), used by the tests and bench.py
  glint_b200.shard       multi-GPU placement: per-tensor LPT and column-parallel
                         linears
  glint_b200.pin         the pin tool (glint_pin.py's interface) as a GPU pipeline
  glint_b200.unpin       the unpin tool (glint_unpin.py's interface) on the GPU
"""
from .build import library_path  # noqa: F401

__version__ = "0.1.0"
