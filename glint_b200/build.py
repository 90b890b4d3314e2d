"""Build libglint_encode.so in-tree (nvcc for sm_100a) and locate it."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

PKG = Path(__file__).resolve().parent
LIB_NAME = "libglint_encode.so"


def library_path() -> Path:
    """GLINT_ENCODE_SO if set (as the reference's glint_cuda.lib_path honours it),
    else the in-tree build."""
    env = os.environ.get("GLINT_ENCODE_SO")
    return Path(env) if env else PKG / LIB_NAME


def build(jobs: int = 4) -> Path:
    """Compile the CUDA library (make -C glint_b200/csrc). Raises on failure."""
    subprocess.run(["make", "-s", "-C", str(PKG / "csrc"), f"-j{jobs}"], check=True)
    p = PKG / LIB_NAME
    if not p.is_file():
        raise RuntimeError(f"build did not produce {p}")
    return p
