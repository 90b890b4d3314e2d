"""glint_htile_stream_noalloc: the decode H-TILE on the library's fixed scratch.

Some callers cannot let a library call cudaMalloc: a serving process whose own
allocator has already taken all free HBM for its cache pool, or an integration
whose device-memory budget is fixed before the first call (a cudaMalloc there can
fail, and it synchronises the device).  For them this entry point runs the decode
kernels with the split-K partial sums and flags in a 4 MiB array compiled into the
library instead of a workspace allocated per stream.

The shapes here are the ones that need that scratch: on 148 SMs, a wide layer past
2 x 112 rows per SM (N = 40960) and narrow layers with long K (N < 16 rows per SM,
K > 8192), which the stream-K kernel serves.  Each is called twice in a row with
different activations, so the second call runs on the flags it re-zeroes and the
partial sums the first call left behind, and each result is checked against the
oracle and against glint_htile_stream, the allocating entry point, within the
tolerances of the other H-TILE tests.  Shapes whose partial sums would not fit the
array must return GLINT_ERR_SCRATCH (-5), which also shows that these shapes reach
the scratch-sizing code.  This file sorts last so that a run that stops at the
first failure has already run every other test.
"""
import ctypes

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import glint_oracle as O  # noqa: E402

PRECISE_TOL = 1e-5
FAST_TOL = 1e-2
SCRATCH_BYTES = 4 << 20
FLAG_BYTES = 64 << 10


def _lib():
    from glint_b200 import build, glint_cuda
    build.build()
    L = glint_cuda.load()
    assert L is not None
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    L.glint_htile_stream_noalloc.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32, i32, i32, vp]
    L.glint_htile_stream_noalloc.restype = i32
    return L


def _rel(y, ref):
    y, ref = y.astype(np.float64), ref.astype(np.float64)
    return float(np.max(np.abs(y - ref)) / max(1.0, float(np.max(np.abs(ref)))))


def _stream_k(sms, N, K):
    """True where the decode takes the stream-K kernel (the one that needs scratch):
    outside the row-owned kernel's range N in [16, 2 * 112 * SMs] with N >= 16 * SMs
    or K <= 8192."""
    return not (16 <= N <= 2 * 112 * sms and (N >= 16 * sms or K <= 8192))


def _scratch_bytes(sms, M, N, K):
    """(flag bytes, partial-sum bytes) a stream-K call needs: row blocks of 256 rows,
    k units of 256 (M <= 16) or 128 (M > 16), MT = 1, 2 or 4 groups of 8 activation
    rows, units split evenly over min(units, SMs) CTAs, at most
    ceil(k units / units per CTA) + 1 parts per row block."""
    MT = 1 if M <= 8 else (2 if M <= 16 else 4)
    ku = K // (256 if MT <= 2 else 128)
    rbs = (N + 255) // 256
    units = rbs * ku
    grid = min(units, sms)
    per_cta = max(1, units // grid)
    parts = min(grid, (ku + per_cta - 1) // per_cta + 1)
    return rbs * parts * 16 * 4, rbs * parts * 256 * 8 * MT * 4


def _fits(sms, M, N, K):
    flags, sums = _scratch_bytes(sms, M, N, K)
    return flags <= FLAG_BYTES and sums <= SCRATCH_BYTES - FLAG_BYTES


@pytest.fixture(scope="module")
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    torch.cuda.set_device(0)
    return _lib(), torch.cuda.get_device_properties(0).multi_processor_count


@pytest.mark.parametrize("M,N,K", [(1, 40960, 4096), (4, 1024, 14336), (1, 1024, 16384), (12, 2048, 16384)])
def test_noalloc_matches_oracle_and_allocating_entry_point(gpu, M, N, K):
    L, sms = gpu
    assert _stream_k(sms, N, K) and _fits(sms, M, N, K), "shape must take the stream-K kernel and fit the array"
    rng = np.random.default_rng(M + N + K)
    w = rng.normal(0, 0.02, N * K).astype(np.float32)
    w[rng.choice(N * K, size=N * K // 1000, replace=False)] *= np.float32(20)
    ho, po, ao = O.encode_bf16(O.f32_to_bf16(w), 64)
    planes = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    assert L.glint_kernel_error(1) == 0
    for call in range(2):
        x_bits = O.f32_to_bf16(rng.normal(0, 1, M * K).astype(np.float32))
        x = torch.from_numpy(x_bits.view(np.int16)).cuda().view(torch.bfloat16).view(M, K)
        ref = O.htile(ho, po, ao, x_bits, M, N, K, 64)
        for mode, tol in ((0, PRECISE_TOL), (1, FAST_TOL)):
            y_ref = torch.empty((M, N), dtype=torch.float32, device="cuda")
            y_new = torch.full((M, N), float("nan"), dtype=torch.float32, device="cuda")
            args = (planes[0].data_ptr(), planes[1].data_ptr(), planes[2].data_ptr(), x.data_ptr())
            assert L.glint_htile_stream(*args, y_ref.data_ptr(), 0, M, N, K, 64, mode, stream) == 0
            assert L.glint_htile_stream_noalloc(*args, y_new.data_ptr(), 0, M, N, K, 64, mode, stream) == 0
            torch.cuda.synchronize()
            assert L.glint_kernel_error(1) == 0
            got, alloc = y_new.cpu().numpy(), y_ref.cpu().numpy()
            assert np.all(np.isfinite(got)), (call, mode)
            assert _rel(got, ref) <= tol, (call, mode, _rel(got, ref))
            assert _rel(got, alloc) <= tol, (call, mode, _rel(got, alloc))
            # the same kernel adds the same parts in the same order
            assert np.array_equal(got, alloc), (call, mode)


def test_noalloc_rejects_what_it_cannot_hold(gpu):
    L, sms = gpu
    z = torch.zeros(1 << 20, dtype=torch.uint8, device="cuda")
    p = z.data_ptr()
    stream = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    # N > 65536 is refused before any size is computed
    assert L.glint_htile_stream_noalloc(p, p, p, p, p, 0, 1, 70000, 256, 64, 0, stream) == -5
    # stream-K shapes whose partial sums exceed the array's 4 MiB - 64 KiB
    for (M, N, K) in ((16, 1024, 16384), (1, 65536, 4096), (32, 40960, 4096)):
        assert _stream_k(sms, N, K) and not _fits(sms, M, N, K)
        assert L.glint_htile_stream_noalloc(p, p, p, p, p, 0, M, N, K, 64, 0, stream) == -5, (M, N, K)
    # shapes outside the decode kernels: blocksize 32, K not a multiple of 256, M > 32
    assert L.glint_htile_stream_noalloc(p, p, p, p, p, 0, 1, 128, 256, 32, 0, stream) == -1
    assert L.glint_htile_stream_noalloc(p, p, p, p, p, 0, 1, 128, 200, 64, 0, stream) == -1
    assert L.glint_htile_stream_noalloc(p, p, p, p, p, 0, 33, 128, 256, 64, 0, stream) == -1
    torch.cuda.synchronize()
    assert L.glint_kernel_error(1) == 0
