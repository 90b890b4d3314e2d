"""The C-ABI library without a GPU: it loads, exports exactly what include/*.h
declares, and rejects bad arguments before touching a device (reference return
codes: cuda/glint_encode.cu:134-262, cuda/glint_htile.cu:170-179)."""
import ctypes
import re
import subprocess
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent


@pytest.fixture(scope="module")
def lib():
    from glint_b200 import build, glint_cuda
    build.build()
    L = glint_cuda.load()
    assert L is not None, glint_cuda._ERR
    return L


def declared_functions():
    names = set()
    for h in (ROOT / "include").glob("*.h"):
        text = re.sub(r"/\*.*?\*/", "", h.read_text(), flags=re.S)
        for m in re.finditer(r"^\s*(?:const\s+)?[A-Za-z_][\w\s\*]*?\b(\w+)\s*\(", text, flags=re.M):
            name = m.group(1)
            if name in ("if", "return", "sizeof") or text[m.start():m.end()].lstrip().startswith("static"):
                continue
            names.add(name)
    return names


def test_library_exports_every_declared_symbol(lib):
    decl = declared_functions()
    assert {"glint_encode_bf16_host", "glint_encode_f32_host", "glint_encode_n_absmax", "glint_encode_n_packed",
            "glint_expand_packed_to_f32_host", "glint_expand_packed_to_f32_device",
            "launch_glint_htile_s3_f32_stream", "launch_glint_htile_s3_f32", "p7_abi_version"} <= decl
    so = ROOT / "glint_b200" / "libglint_encode.so"
    out = subprocess.run(["nm", "-D", "--defined-only", str(so)], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    assert decl <= exported, sorted(decl - exported)
    # only the C ABI leaves the library (kernels and C++ helpers stay local)
    assert all(s.startswith(("glint_", "launch_glint_htile_", "int8_mma_gemm", "p7_abi_version")) for s in exported), \
        exported


def test_attach_abi_version(lib):
    assert lib.p7_abi_version() == b"p7_attach_abi_v1"
    assert lib.glint_b200_version().startswith(b"glint_b200 ")


def test_size_helpers_match_reference(lib):
    # glint_encode.cu:128-133: ceil(n/bs) (0 for bs <= 0) and ceil(n/2), as int
    for n, bs in [(0, 64), (1, 64), (64, 64), (65, 64), (16777216, 64), (7, 23), (5, 0), (5, -3)]:
        assert lib.glint_encode_n_absmax(n, bs) == ((n + bs - 1) // bs if bs > 0 else 0)
        assert lib.glint_encode_n_packed(n) == (n + 1) // 2
    assert lib.glint_encode_n_absmax64(1 << 40, 64) == (1 << 40) // 64
    assert lib.glint_encode_n_packed64((1 << 40) + 1) == (1 << 39) + 1


def test_bad_arguments_rejected_without_gpu(lib):
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    assert lib.glint_encode_bf16_host(p, 4, 0, p, p, p) == -1          # blocksize <= 0
    assert lib.glint_encode_bf16_host(p, -1, 64, p, p, p) == -1        # n < 0
    assert lib.glint_encode_bf16_host(None, 4, 64, p, p, p) == -1      # null
    assert lib.glint_encode_bf16_host(p, 0, 64, p, p, p) == 0          # nothing to do
    assert lib.glint_expand_packed_to_f32_device(None, p, p, 4, 64, p, None) == -1
    assert lib.glint_expand_packed_to_f32_device(p, p, p, 4, 0, p, None) == -1
    assert lib.glint_expand_packed_to_f32_device(p, p, p, 0, 64, p, None) == 0
    assert lib.launch_glint_htile_s3_f32(None, p, p, p, p, 1, 1, 1, 64) == -1
    assert lib.launch_glint_htile_s3_f32(p, p, p, p, p, 1, 1, 1, 0) == -2
    assert lib.launch_glint_htile_s3_f32(p, p, p, p, p, 0, 5, 5, 64) == 0
    assert lib.glint_htile_stream(p, p, p, p, p, 7, 1, 1, 1, 64, 0, None) == -1   # bad y dtype
    assert lib.glint_htile_stream(p, p, p, p, p, 0, 1, 1, 1, 64, 9, None) == -1   # bad mode


def test_codebook_export_and_sqerr_arguments_without_gpu(lib):
    """glint_cells_f32 returns the pinned codebook (the bits the reference's
    glint_codec.CELLS holds, tests/golden/tables.json) with no GPU; the
    glint_encode_*_host_sqerr entries check their arguments before any device work
    and give a zero sum for an empty tensor."""
    import json
    import numpy as np
    cells = np.empty(256, dtype="<f4")
    assert lib.glint_cells_f32(cells.ctypes.data) == 256
    want = json.loads((ROOT / "tests" / "golden" / "tables.json").read_text())["cells_bits"]
    assert cells.view("<u4").tolist() == want
    assert lib.glint_cells_f32(None) == -1
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    sq = ctypes.c_double(-1.0)
    for f in (lib.glint_encode_bf16_host_sqerr, lib.glint_encode_f32_host_sqerr):
        assert f(p, 4, 64, p, p, p, None) == -1                       # no sum pointer
        assert f(p, -1, 64, p, p, p, ctypes.byref(sq)) == -1          # n < 0
        assert f(p, 4, 0, p, p, p, ctypes.byref(sq)) == -1            # blocksize <= 0
        assert f(None, 4, 64, p, p, p, ctypes.byref(sq)) == -1        # null input
        sq.value = -1.0
        assert f(p, 0, 64, p, p, p, ctypes.byref(sq)) == 0 and sq.value == 0.0   # empty tensor


def test_gathered_decode_and_ipc_reject_bad_arguments_without_gpu(lib):
    """glint_htile_gather_stream and the IPC helpers check their arguments before
    touching a device (include/glint_htile.h; -1 bad argument, -2 blocksize)."""
    buf = (ctypes.c_uint8 * 64)()
    p = ctypes.addressof(buf)
    ptrs = (ctypes.c_void_p * 2)(p, p)
    nul = (ctypes.c_void_p * 2)(p, None)
    g = lib.glint_htile_gather_stream
    assert g(None, p, p, p, ptrs, ptrs, 2, 0, 0, 1, 64, 256, 128, 0, 64, 1, None) == -1   # null plane
    assert g(p, p, p, p, nul, ptrs, 2, 0, 0, 1, 64, 256, 128, 0, 64, 1, None) == -1       # null peer y
    assert g(p, p, p, p, ptrs, nul, 2, 0, 0, 1, 64, 256, 128, 0, 64, 1, None) == -1       # null peer counters
    assert g(p, p, p, p, ptrs, ptrs, 2, 2, 0, 1, 64, 256, 128, 0, 64, 1, None) == -1      # rank >= world
    assert g(p, p, p, p, ptrs, ptrs, 2, 0, 5, 1, 64, 256, 128, 0, 64, 1, None) == -1      # bad y dtype
    assert g(p, p, p, p, ptrs, ptrs, 2, 0, 0, 1, 64, 256, 128, 0, 64, 7, None) == -1      # bad mode
    assert g(p, p, p, p, ptrs, ptrs, 2, 0, 0, 1, 64, 256, 128, 0, 0, 1, None) == -2       # blocksize
    assert g(p, p, p, p, ptrs, ptrs, 2, 0, 0, 1, 64, 256, 100, 64, 64, 1, None) == -1     # rows past ld_y
    q = ctypes.c_void_p()
    assert lib.glint_device_alloc(0, ctypes.byref(q)) == -1
    assert lib.glint_ipc_handle(None, p) == -1
    assert lib.glint_ipc_open(None, ctypes.byref(q)) == -1
    assert lib.glint_ipc_close(None) == -1


def test_headers_compile_and_link_from_plain_c(lib, tmp_path):
    """Every public header compiles in a C11 translation unit and the library links
    from C (tests/native/abi_from_c.c); the device-free helpers answer."""
    import shutil
    if shutil.which("gcc") is None:
        pytest.skip("gcc absent")
    exe = tmp_path / "abi_from_c"
    cuda_inc = "/usr/local/cuda/include"
    subprocess.run(["gcc", "-std=c11", "-Wall", "-Wextra", "-Werror", f"-I{cuda_inc}", "-o", str(exe),
                    str(ROOT / "tests" / "native" / "abi_from_c.c"), f"-L{ROOT / 'glint_b200'}", "-lglint_encode",
                    f"-Wl,-rpath,{ROOT / 'glint_b200'}"], check=True)
    r = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert r.returncode == 0 and r.stdout.strip() == "OK", r.stdout + r.stderr


def test_glint_cuda_mirror_interface():
    """Same public names and signatures as the reference's glint_cuda.py:1-85."""
    import inspect
    from glint_b200 import glint_cuda as G
    for name in ("lib_path", "load", "encode_bf16_cuda", "expand_cuda", "gpu_ok"):
        assert callable(getattr(G, name))
    assert list(inspect.signature(G.encode_bf16_cuda).parameters) == ["raw_bf16", "n", "blocksize"]
    assert list(inspect.signature(G.expand_cuda).parameters) == ["hole", "plug", "absmax_f32", "n", "blocksize"]
