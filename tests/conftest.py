"""Shared pytest setup: the `gpu` marker and import paths.

`-m "not gpu"` runs here without a GPU: oracle vs golden vectors, host logic,
the C-ABI library's symbol table.  `-m gpu` is the parity suite proper and calls
the CUDA library through its C ABI on a B200.
"""
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent.parent
for p in (ROOT, ROOT / "oracle"):
    if str(p) not in sys.path:
        sys.path.insert(0, str(p))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libglint_encode.so")
