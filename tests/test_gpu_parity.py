"""GPU parity: libglint_encode.so through its C ABI against the CPU oracle, the
golden vectors written from the reference, and the reference's own kernels
built for sm_100a (oracle/_ref, when present).

Bars (north star): encode bytes and expanded BF16 bit-exact; H-TILE within
max|y - y_ref| <= 1e-2 * max(1, max|y_ref|) of an f32 dequant-then-matmul in
fast mode, and within the reference's own device-test bound
1e-5 * (1 + |ref|) (tests/test_htile_k_bounds_device.cu:98) in precise mode.
"""
import ctypes
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import glint_oracle as O  # noqa: E402

G = Path(__file__).resolve().parent / "golden"
PRECISE_TOL = 1e-5
FAST_TOL = 1e-2


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from glint_b200 import build
    build.build()
    O.set_threads()
    torch.cuda.set_device(0)


def D():
    from glint_b200 import device
    return device


def synth_bf16(n, seed=0, outliers=0.001):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, n).astype(np.float32)
    k = int(outliers * n)
    if k:
        w[rng.choice(n, size=k, replace=False)] *= np.float32(20)
    return O.f32_to_bf16(w)


def to_dev_bf16(bits: np.ndarray):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def host_bytes(t):
    return t.cpu().numpy().tobytes()


def golden_names(npz):
    d = np.load(G / npz)
    return sorted({k.split("__")[0] for k in d.files})


# ---------------------------------------------------------------- encode
@pytest.mark.parametrize("name", golden_names("encode_bf16.npz"))
def test_encode_bf16_matches_golden(name):
    d = np.load(G / "encode_bf16.npz")
    bs = int(d[name + "__bs"][0])
    h, p, a = D().encode(to_dev_bf16(d[name + "__w"]), bs)
    torch.cuda.synchronize()
    assert host_bytes(h) == d[name + "__hole"].tobytes()
    assert host_bytes(p) == d[name + "__plug"].tobytes()
    assert host_bytes(a) == d[name + "__absmax"].tobytes()


@pytest.mark.parametrize("name", golden_names("encode_f32.npz"))
def test_encode_f32_matches_golden(name):
    d = np.load(G / "encode_f32.npz")
    bs = int(d[name + "__bs"][0])
    h, p, a = D().encode(torch.from_numpy(d[name + "__w"]).cuda(), bs)
    torch.cuda.synchronize()
    assert host_bytes(h) == d[name + "__hole"].tobytes()
    assert host_bytes(p) == d[name + "__plug"].tobytes()
    assert host_bytes(a) == d[name + "__absmax"].tobytes()


def test_encode_host_abi_matches_golden():
    """glint_encode_bf16_host via the reference-shaped ctypes wrapper (glint_cuda.py:52-65)."""
    from glint_b200 import glint_cuda
    assert glint_cuda.gpu_ok()
    d = np.load(G / "encode_bf16.npz")
    for name in golden_names("encode_bf16.npz"):
        bs = int(d[name + "__bs"][0])
        w = d[name + "__w"]
        h, p, a = glint_cuda.encode_bf16_cuda(w.tobytes(), w.size, bs)
        assert h == d[name + "__hole"].tobytes(), name
        assert p == d[name + "__plug"].tobytes(), name
        assert a == d[name + "__absmax"].tobytes(), name


def test_encode_batch_matches_single():
    d = np.load(G / "encode_bf16.npz")
    names = [n for n in golden_names("encode_bf16.npz") if int(d[n + "__bs"][0]) == 64]
    ws = [to_dev_bf16(d[n + "__w"]) for n in names]
    outs = D().encode_batch(ws, 64)
    torch.cuda.synchronize()
    for n, (h, p, a) in zip(names, outs):
        assert host_bytes(h) == d[n + "__hole"].tobytes(), n
        assert host_bytes(p) == d[n + "__plug"].tobytes(), n
        assert host_bytes(a) == d[n + "__absmax"].tobytes(), n


@pytest.mark.parametrize("bs", [8, 16, 32, 64, 128, 256, 1, 23, 96, 512])
@pytest.mark.parametrize("n", [1, 2, 255, 256, 257, 4097, 100003])
def test_encode_ragged_sizes_vs_oracle(n, bs):
    bits = synth_bf16(n, seed=n * 31 + bs)
    h, p, a = D().encode(to_dev_bf16(bits), bs)
    ho, po, ao = O.encode_bf16(bits, bs)
    torch.cuda.synchronize()
    assert host_bytes(h) == ho.tobytes()
    assert host_bytes(p) == po.tobytes()
    assert host_bytes(a) == ao.tobytes()


@pytest.mark.parametrize("shift", [1, 3, 8])
def test_encode_unaligned_pointers(shift):
    """Views that start off a 16-byte boundary take the generic path."""
    n, bs = 50001, 64
    bits = synth_bf16(n + shift, seed=shift)
    base = to_dev_bf16(bits)
    w = base[shift:]
    hb = torch.zeros(n // 2 + 8, dtype=torch.uint8, device="cuda")
    pb = torch.zeros_like(hb)
    ab = torch.zeros(n // bs + 8, dtype=torch.float32, device="cuda")
    h, p, a = hb[1:1 + (n + 1) // 2], pb[1:1 + (n + 1) // 2], ab[1:1 + (n + bs - 1) // bs]
    D().encode(w, bs, out=(h, p, a))
    ho, po, ao = O.encode_bf16(bits[shift:], bs)
    torch.cuda.synchronize()
    assert host_bytes(h) == ho.tobytes() and host_bytes(p) == po.tobytes() and host_bytes(a) == ao.tobytes()
    assert hb[0].item() == 0 and pb[0].item() == 0 and ab[0].item() == 0  # nothing written before the view


def test_encode_config1_tensor_vs_oracle():
    """Config 1: one 4096x4096 N(0,0.02) + 0.1% x20 BF16 weight, bs 64."""
    n = 4096 * 4096
    bits = synth_bf16(n, seed=0)
    h, p, a = D().encode(to_dev_bf16(bits), 64)
    ho, po, ao = O.encode_bf16(bits, 64)
    torch.cuda.synchronize()
    assert host_bytes(h) == ho.tobytes()
    assert host_bytes(p) == po.tobytes()
    assert host_bytes(a) == ao.tobytes()


def test_encode_adversarial_blocks_vs_oracle():
    """2^22 blocks whose absmax and members are arbitrary BF16 bit patterns
    (every exponent, denormals, NaN, inf), so the divide sees every regime."""
    rng = np.random.default_rng(7)
    nblk = 1 << 16
    w = rng.integers(0, 1 << 16, size=(nblk, 64), dtype=np.uint32).astype(np.uint16)
    # in half the blocks shrink members below a chosen max to exercise |w| <= s near 1
    lead = rng.integers(0, 0x7F80, size=nblk, dtype=np.uint32).astype(np.uint16)
    half = nblk // 2
    w[:half, 0] = lead[:half]
    mag = w[:half, 1:] & 0x7FFF
    w[:half, 1:] = np.where(mag > lead[:half, None], lead[:half, None] - (mag % 16), w[:half, 1:]) | (w[:half, 1:] & 0x8000)
    bits = w.reshape(-1)
    h, p, a = D().encode(to_dev_bf16(bits), 64)
    ho, po, ao = O.encode_bf16(bits, 64)
    torch.cuda.synchronize()
    assert host_bytes(h) == ho.tobytes()
    assert host_bytes(p) == po.tobytes()
    assert host_bytes(a) == ao.tobytes()


def test_encode_host_pipeline_multi_chunk():
    """n spans several 16 Mi-weight pipeline chunks with a ragged end, from pinned
    and from pageable host memory; equals the device entry point byte for byte."""
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    n = 3 * (1 << 24) + 12345
    bits = synth_bf16(n, seed=5)
    ho, po, ao = O.encode_bf16(bits, 64)
    for pinned in (True, False):
        src = torch.from_numpy(bits.view(np.int16))
        hole = torch.empty((n + 1) // 2, dtype=torch.uint8)
        plug = torch.empty_like(hole)
        am = torch.empty((n + 63) // 64, dtype=torch.float32)
        if pinned:
            src, hole, plug, am = src.pin_memory(), hole.pin_memory(), plug.pin_memory(), am.pin_memory()
        rc = L.glint_encode_bf16_host(src.data_ptr(), n, 64, hole.data_ptr(), plug.data_ptr(), am.data_ptr())
        assert rc == 0
        assert hole.numpy().tobytes() == ho.tobytes(), pinned
        assert plug.numpy().tobytes() == po.tobytes(), pinned
        assert am.numpy().tobytes() == ao.tobytes(), pinned


def test_encode_matches_reference_library():
    """Byte parity with the reference's own libglint_encode.so built for sm_100a."""
    so = O.ref_lib_path("libglint_encode.so")
    if so is None:
        pytest.skip("oracle/_ref not built")
    R = ctypes.CDLL(str(so))
    vp = ctypes.c_void_p
    R.glint_encode_bf16_host.argtypes = [vp, ctypes.c_int64, ctypes.c_int, vp, vp, vp]
    for n, bs, seed in [(4096 * 1024, 64, 1), (100003, 23, 2), (65536, 64, 3)]:
        bits = synth_bf16(n, seed=seed)
        if seed == 3:
            bits = np.random.default_rng(3).permutation(np.arange(65536, dtype=np.uint32)).astype(np.uint16)
        hr = np.zeros((n + 1) // 2, np.uint8)
        pr = np.zeros_like(hr)
        ar = np.zeros((n + bs - 1) // bs, np.float32)
        assert R.glint_encode_bf16_host(bits.ctypes.data, n, bs, hr.ctypes.data, pr.ctypes.data, ar.ctypes.data) == 0
        h, p, a = D().encode(to_dev_bf16(bits), bs)
        torch.cuda.synchronize()
        assert host_bytes(h) == hr.tobytes()
        assert host_bytes(p) == pr.tobytes()
        assert host_bytes(a) == ar.tobytes()


# ---------------------------------------------------------------- expand
def test_expand_specials_match_golden():
    d = np.load(G / "expand.npz")
    n, bs = int(d["n"][0]), int(d["bs"][0])
    hole, plug, am = (torch.from_numpy(d[k]).cuda() for k in ("hole", "plug", "absmax"))
    yb = D().expand(hole, plug, am, n, bs, torch.bfloat16)
    yf = D().expand(hole, plug, am, n, bs, torch.float32)
    torch.cuda.synchronize()
    assert host_bytes(yb.view(torch.int16)) == d["expand_bf16"].tobytes()
    assert host_bytes(yf) == d["expand_f32"].tobytes()


@pytest.mark.parametrize("name", golden_names("encode_bf16.npz"))
def test_expand_matches_golden(name):
    d = np.load(G / "encode_bf16.npz")
    bs = int(d[name + "__bs"][0])
    n = d[name + "__w"].size
    hole, plug, am = (torch.from_numpy(d[name + k]).cuda() for k in ("__hole", "__plug", "__absmax"))
    yb = D().expand(hole, plug, am, n, bs, torch.bfloat16)
    yf = D().expand(hole, plug, am, n, bs, torch.float32)
    torch.cuda.synchronize()
    assert host_bytes(yb.view(torch.int16)) == d[name + "__expand_bf16"].tobytes()
    assert host_bytes(yf) == d[name + "__expand_f32"].tobytes()


def test_expand_host_abi_matches_golden():
    from glint_b200 import glint_cuda
    d = np.load(G / "encode_bf16.npz")
    for name in golden_names("encode_bf16.npz"):
        bs = int(d[name + "__bs"][0])
        n = d[name + "__w"].size
        args = (d[name + "__hole"].tobytes(), d[name + "__plug"].tobytes(), d[name + "__absmax"].tobytes(), n, bs)
        assert glint_cuda.expand_cuda(*args) == d[name + "__expand_f32"].tobytes(), name
        assert glint_cuda.expand_bf16_cuda(*args) == d[name + "__expand_bf16"].tobytes(), name


@pytest.mark.parametrize("bs", [8, 64, 128, 23, 1, 96])
@pytest.mark.parametrize("n", [1, 255, 257, 100003, 3 * (1 << 20) + 7])
def test_expand_random_vs_oracle(n, bs):
    rng = np.random.default_rng(n + bs)
    hole = rng.integers(0, 256, (n + 1) // 2, dtype=np.uint8)
    plug = rng.integers(0, 256, (n + 1) // 2, dtype=np.uint8)
    am = np.abs(rng.normal(0, 0.05, (n + bs - 1) // bs)).astype(np.float32)
    yb = D().expand(*(torch.from_numpy(a).cuda() for a in (hole, plug, am)), n, bs, torch.bfloat16)
    yf = D().expand(*(torch.from_numpy(a).cuda() for a in (hole, plug, am)), n, bs, torch.float32)
    torch.cuda.synchronize()
    assert host_bytes(yb.view(torch.int16)) == O.expand_bf16(hole, plug, am, n, bs).tobytes()
    assert host_bytes(yf) == O.expand_f32(hole, plug, am, n, bs).tobytes()


def test_expand_batch_and_host_pipeline():
    from glint_b200 import glint_cuda
    sizes = [4096 * 1024, 1024 * 4096 + 3, 1, 777]
    planes, outs, refs = [], [], []
    for i, n in enumerate(sizes):
        bits = synth_bf16(n, seed=40 + i)
        ho, po, ao = O.encode_bf16(bits, 64)
        planes.append(tuple(torch.from_numpy(a).cuda() for a in (ho, po, ao)))
        outs.append(torch.empty(n, dtype=torch.bfloat16, device="cuda"))
        refs.append((ho, po, ao, O.expand_bf16(ho, po, ao, n, 64)))
    D().expand_batch(planes, outs, 64)
    torch.cuda.synchronize()
    for o, r in zip(outs, refs):
        assert host_bytes(o.view(torch.int16)) == r[3].tobytes()
    n = 2 * (1 << 24) + 99
    bits = synth_bf16(n, seed=9)
    ho, po, ao = O.encode_bf16(bits, 64)
    got = glint_cuda.expand_bf16_cuda(ho.tobytes(), po.tobytes(), ao.tobytes(), n, 64)
    assert got == O.expand_bf16(ho, po, ao, n, 64).tobytes()


# ---------------------------------------------------------------- H-TILE
def rel_err(y, ref):
    return float(np.max(np.abs(y.astype(np.float64) - ref)) / max(1.0, float(np.max(np.abs(ref)))))


@pytest.mark.parametrize("key", golden_names("htile.npz"))
def test_htile_matches_reference_sim(key):
    d = np.load(G / "htile.npz")
    M, N, K, bs = (int(v) for v in d[key + "__shape"])
    hole, plug, am = (torch.from_numpy(d[key + k]).cuda() for k in ("__hole", "__plug", "__absmax"))
    x = to_dev_bf16(d[key + "__x"]).view(M, K)
    ref = d[key + "__y"].reshape(M, N)
    y = D().htile_reference_abi(x, hole, plug, am, N, bs)
    yf = D().htile(x, hole, plug, am, N, bs, mode="fast")
    torch.cuda.synchronize()
    y, yf = y.cpu().numpy(), yf.cpu().numpy()
    assert np.all(np.abs(y - ref) <= PRECISE_TOL * (1 + np.abs(ref)))
    assert rel_err(yf, ref) <= FAST_TOL


def _k_bounds_case(M, N, K, bs):
    """Inputs of tests/test_htile_k_bounds_device.cu:53-67 (patterned codes, scales, x)."""
    i = np.arange(N * K)
    h = ((i * 7 + i // 17 + 3) % 16).astype(np.uint8)
    p = ((i * 11 + i // 13 + 5) % 16).astype(np.uint8)
    npk = (N * K + 1) // 2
    hole = np.zeros(npk, np.uint8)
    plug = np.zeros(npk, np.uint8)
    np.bitwise_or.at(hole, i // 2, (h << (4 * (i % 2))).astype(np.uint8))
    np.bitwise_or.at(plug, i // 2, (p << (4 * (i % 2))).astype(np.uint8))
    nb = (N * K + bs - 1) // bs
    am = (0.25 + (np.arange(nb) % 7) * 0.125).astype(np.float32)
    j = np.arange(M * K)
    x = O.f32_to_bf16(((((j * 3 + j // 19) % 17) - 8) * 0.0625).astype(np.float32))
    return hole, plug, am, x


@pytest.mark.parametrize("shift", [0, 1])
def test_htile_k_bounds_misaligned_canaries(shift):
    """The reference's device bounds test: K tails, blocksize 23 straddling rows,
    pointers shifted off alignment, canaries around y, three repetitions."""
    bs, guard, canary = 23, 16, 123456.0
    for K in (1, 32, 40, 48, 63, 64, 65, 192, 199, 256):
        for (M, N) in ((1, 1), (15, 15), (16, 16), (17, 19), (33, 31)):
            hole, plug, am, x = _k_bounds_case(M, N, K, bs)
            ref = O.htile(hole, plug, am, x, M, N, K, bs).astype(np.float64)

            def shifted(a, dtype):
                base = torch.zeros(a.size + shift, dtype=dtype, device="cuda")
                base[shift:] = torch.from_numpy(a.view(np.int16) if dtype == torch.int16 else a).cuda()
                return base[shift:]
            dh, dp = shifted(hole, torch.uint8), shifted(plug, torch.uint8)
            dx = shifted(x, torch.int16).view(torch.bfloat16).view(M, K)
            da = torch.from_numpy(am).cuda()
            ybuf = torch.full((M * N + 2 * guard,), canary, dtype=torch.float32, device="cuda")
            for _ in range(3):
                y = ybuf[guard:guard + M * N].view(M, N)
                D().htile_reference_abi(dx, dh, dp, da, N, bs, out=y)
                torch.cuda.synchronize()
                yb = ybuf.cpu().numpy()
                assert np.all(yb[:guard] == canary) and np.all(yb[guard + M * N:] == canary), (M, N, K)
                got = yb[guard:guard + M * N].reshape(M, N).astype(np.float64)
                assert np.all(np.isfinite(got))
                assert np.all(np.abs(got - ref) <= PRECISE_TOL * (1 + np.abs(ref))), (M, N, K, shift)


@pytest.mark.parametrize("M,N,K", [(16, 16, 64), (16, 16, 128), (32, 32, 192), (16, 16, 32), (16, 16, 48),
                                   (16, 16, 40), (16, 16, 70), (16, 16, 100), (7, 23, 64), (4, 3072, 3072)])
def test_htile_reference_shapes(M, N, K):
    """Shapes and data of tests/test_glint_htile.cu:63-74,135-162 (tolerance 1e-3 there)."""
    bs = 64
    npk, nam = (N * K + 1) // 2, (N * K + bs - 1) // bs
    i = np.arange(npk)
    hole = ((i * 7 + 1) % 256).astype(np.uint8)
    plug = ((i * 13 + 5) % 256).astype(np.uint8)
    am = (0.5 + (np.arange(nam) % 10) * 0.1).astype(np.float32)
    j = np.arange(M * K)
    x = O.f32_to_bf16(((((j * 17 + 3) % 100) - 50.0) * 0.01).astype(np.float32))
    ref = O.htile(hole, plug, am, x, M, N, K, bs).astype(np.float64)
    y = D().htile_reference_abi(to_dev_bf16(x).view(M, K), *(torch.from_numpy(a).cuda() for a in (hole, plug, am)),
                                N, bs)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    assert np.max(np.abs(got - ref)) < 1e-3
    # f32-class accuracy measured against the sum's own scale sum_k |w x| (heavy cancellation here)
    W = O.expand_f32(hole, plug, am, N * K, bs).reshape(N, K).astype(np.float64)
    scale = np.abs(O.bf16_to_f32(x).reshape(M, K).astype(np.float64)) @ np.abs(W).T
    assert np.all(np.abs(got - ref) <= 1e-6 * (1 + scale))


@pytest.mark.parametrize("M", [1, 4, 16])
@pytest.mark.parametrize("K,N", [(4096, 14336), (14336, 4096)])
def test_htile_decode_config3(M, K, N):
    """Config 3 decode shapes: fast within 1e-2 relative, precise within 1e-5 relative."""
    bits = synth_bf16(N * K, seed=M + K)
    ho, po, ao = O.encode_bf16(bits, 64)
    rng = np.random.default_rng(M)
    x = O.f32_to_bf16(rng.normal(0, 1, M * K).astype(np.float32))
    ref = O.htile(ho, po, ao, x, M, N, K, 64).astype(np.float64)
    dev = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
    dx = to_dev_bf16(x).view(M, K)
    yp = D().htile(dx, *dev, N, 64, mode="precise").cpu().numpy()
    yf = D().htile(dx, *dev, N, 64, mode="fast").cpu().numpy()
    yb = D().htile(dx, *dev, N, 64, mode="fast", out_dtype=torch.bfloat16).float().cpu().numpy()
    assert rel_err(yp, ref) <= PRECISE_TOL
    assert rel_err(yf, ref) <= FAST_TOL
    assert rel_err(yb, ref) <= FAST_TOL


def test_htile_matches_reference_library():
    """Same inputs through the reference's launch_glint_htile_s3_f32 (sm_100a build)."""
    so = O.ref_lib_path("libglint_htile.so")
    if so is None:
        pytest.skip("oracle/_ref not built")
    R = ctypes.CDLL(str(so))
    vp, i32 = ctypes.c_void_p, ctypes.c_int
    R.launch_glint_htile_s3_f32.argtypes = [vp, vp, vp, vp, vp, i32, i32, i32, i32]
    for (M, N, K, bs) in [(4, 512, 1024, 64), (17, 33, 199, 23), (64, 256, 512, 64)]:
        bits = synth_bf16(N * K, seed=N)
        ho, po, ao = O.encode_bf16(bits, bs)
        x = O.f32_to_bf16(np.random.default_rng(K).normal(0, 1, M * K).astype(np.float32))
        dev = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
        dx = to_dev_bf16(x).view(M, K)
        yr = torch.empty((M, N), dtype=torch.float32, device="cuda")
        assert R.launch_glint_htile_s3_f32(*(t.data_ptr() for t in dev[:2]), dev[2].data_ptr(), dx.data_ptr(),
                                           yr.data_ptr(), M, N, K, bs) == 0
        y = D().htile_reference_abi(dx, *dev, N, bs)
        torch.cuda.synchronize()
        ref = yr.cpu().numpy().astype(np.float64)
        assert np.all(np.abs(y.cpu().numpy() - ref) <= 2 * PRECISE_TOL * (1 + np.abs(ref)))


@pytest.mark.parametrize("M,N,K", [(128, 256, 64), (256, 256, 4096), (300, 200, 128), (129, 264, 192),
                                   (512, 512, 1024), (1024, 512, 4096), (256, 4096, 256), (300, 200, 256),
                                   (129, 264, 512), (640, 1000, 768), (2048, 384, 1024), (1100, 130, 2048),
                                   (256, 512, 4096), (384, 4608, 1280)])
def test_htile_prefill_tcgen05_vs_oracle(M, N, K):
    """Prefill shapes take the tcgen05 path: fast mode within 1e-2 relative of the f32
    dequant-then-matmul oracle, precise mode (and the reference ABI) within 1e-5, f32 and
    BF16 y, ragged M and N edges, tiles split between 1 to 16 CTA pairs, bit-identical
    repeated calls."""
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    assert L.glint_kernel_error(1) == 0
    bits = synth_bf16(N * K, seed=M * 7 + N)
    ho, po, ao = O.encode_bf16(bits, 64)
    x = O.f32_to_bf16(np.random.default_rng(M + K).normal(0, 1, M * K).astype(np.float32))
    ref = O.htile(ho, po, ao, x, M, N, K, 64).astype(np.float64)
    dev = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
    dx = to_dev_bf16(x).view(M, K)
    yt = D().htile(dx, *dev, N, 64, mode="fast")
    yt2 = D().htile(dx, *dev, N, 64, mode="fast")
    yf = yt.cpu().numpy()
    yb = D().htile(dx, *dev, N, 64, mode="fast", out_dtype=torch.bfloat16).float().cpu().numpy()
    assert L.glint_kernel_error(1) == 0
    assert torch.equal(yt, yt2)  # split tiles are summed in a fixed order
    assert np.all(np.isfinite(yf))
    assert rel_err(yf, ref) <= FAST_TOL, rel_err(yf, ref)
    assert rel_err(yb, ref) <= FAST_TOL, rel_err(yb, ref)
    # precise mode (hi + lo halves on the tensor cores) and the reference ABI, which is precise
    yp = D().htile(dx, *dev, N, 64, mode="precise")
    yp2 = D().htile(dx, *dev, N, 64, mode="precise")
    yr = D().htile_reference_abi(dx, *dev, N, 64)
    torch.cuda.synchronize()
    assert L.glint_kernel_error(1) == 0
    assert torch.equal(yp, yp2)
    assert rel_err(yp.cpu().numpy(), ref) <= PRECISE_TOL, rel_err(yp.cpu().numpy(), ref)
    assert rel_err(yr.cpu().numpy(), ref) <= PRECISE_TOL, rel_err(yr.cpu().numpy(), ref)


_FULL_PLANES = {}


def _full_size_planes(N, K):
    """Planes of one [N, K] weight drawn as the prefill config draws them (N(0, 0.02),
    exactly 0.1 % of entries x20 without replacement, BF16 RNE), encoded by the oracle;
    cached per shape so the six shapes encode two weights."""
    if (N, K) not in _FULL_PLANES:
        _FULL_PLANES.clear()
        bits = synth_bf16(N * K, seed=N + K)
        ho, po, ao = O.encode_bf16(bits, 64)
        _FULL_PLANES[(N, K)] = (ho, po, ao, [torch.from_numpy(a).cuda() for a in (ho, po, ao)])
    return _FULL_PLANES[(N, K)]


def _sample_rows(M, count=64):
    """count rows of an M-row activation: both ends, the 128/256-row tile edges and
    evenly spread rows between them (y row m depends on x row m only)."""
    edges = {0, 1, 127, 128, 255, 256, M // 2, M - 2, M - 1}
    spread = np.linspace(0, M - 1, count - len(edges)).astype(np.int64)
    return np.array(sorted(edges.union(spread.tolist())), np.int64)[:count]


@pytest.mark.parametrize("N", [4096, 14336])
@pytest.mark.parametrize("M", [512, 2048, 8192])
def test_htile_prefill_full_config_vs_oracle(M, N):
    """The prefill config at its full sizes (M in {512, 2048, 8192}, K = 4096,
    N in {4096, 14336}): the tcgen05 kernel's full-size schedules (data-parallel
    rounds and the stream-K remainder over 56 to 448 tiles per CTA pair) in fast mode
    within max|y - y_ref| <= 1e-2 * max(1, max|y_ref|) of the oracle on a 64-row
    sample of y (the oracle computes the sampled rows only), BF16 y too, and two
    calls bit-identical."""
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    K = 4096
    ho, po, ao, dev = _full_size_planes(N, K)
    x = O.f32_to_bf16(np.random.default_rng(M + N).normal(0, 1, M * K).astype(np.float32)).reshape(M, K)
    rows = _sample_rows(M)
    ref = O.htile(ho, po, ao, np.ascontiguousarray(x[rows]), len(rows), N, K, 64).astype(np.float64)
    dx = to_dev_bf16(x.reshape(-1)).view(M, K)
    yf = D().htile(dx, *dev, N, 64, mode="fast")
    yf2 = D().htile(dx, *dev, N, 64, mode="fast")
    yb = D().htile(dx, *dev, N, 64, mode="fast", out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert L.glint_kernel_error(1) == 0
    assert torch.equal(yf, yf2)
    idx = torch.from_numpy(rows).cuda()
    got = yf.index_select(0, idx).cpu().numpy()
    gotb = yb.index_select(0, idx).float().cpu().numpy()
    assert np.all(np.isfinite(got))
    assert rel_err(got, ref) <= FAST_TOL, rel_err(got, ref)
    assert rel_err(gotb, ref) <= FAST_TOL, rel_err(gotb, ref)
    # the reference's own entry point (precise: the cell as BF16 hi + lo, a fresh
    # tensor-core accumulator per 64-k block, the blocks scaled and added in f32)
    # within 1e-5 of max(1, max|ref|), as the other precise checks at long K
    yr = D().htile_reference_abi(dx, *dev, N, 64)
    yr2 = D().htile_reference_abi(dx, *dev, N, 64)
    torch.cuda.synchronize()
    assert L.glint_kernel_error(1) == 0
    assert torch.equal(yr, yr2)
    gotr = yr.index_select(0, idx).cpu().numpy()
    assert rel_err(gotr, ref) <= PRECISE_TOL, rel_err(gotr, ref)


@pytest.mark.parametrize("M,N,K", [(1, 100, 256), (3, 1000, 512), (16, 4096, 14336), (17, 384, 2048), (32, 200, 4096),
                                   (5, 14336, 4096), (2, 130, 768)])
def test_htile_decode_stream_k_vs_oracle(M, N, K):
    """Decode shapes on the TMA-streamed stream-K kernel: ragged N, single-unit K,
    row blocks split across CTAs; precise within 1e-5, fast within 1e-2, and two
    calls give identical bits (the split parts are added in a fixed order)."""
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    bits = synth_bf16(N * K, seed=N + K + M)
    ho, po, ao = O.encode_bf16(bits, 64)
    x = O.f32_to_bf16(np.random.default_rng(M * N).normal(0, 1, M * K).astype(np.float32))
    ref = O.htile(ho, po, ao, x, M, N, K, 64).astype(np.float64)
    dev = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
    dx = to_dev_bf16(x).view(M, K)
    yp = D().htile(dx, *dev, N, 64, mode="precise")
    yp2 = D().htile(dx, *dev, N, 64, mode="precise")
    yf = D().htile(dx, *dev, N, 64, mode="fast")
    yb = D().htile(dx, *dev, N, 64, mode="fast", out_dtype=torch.bfloat16)
    torch.cuda.synchronize()
    assert L.glint_kernel_error(1) == 0
    assert torch.equal(yp, yp2)
    assert rel_err(yp.cpu().numpy(), ref) <= PRECISE_TOL
    assert rel_err(yf.cpu().numpy(), ref) <= FAST_TOL
    assert rel_err(yb.float().cpu().numpy(), ref) <= FAST_TOL


@pytest.mark.parametrize("M,N,K", [(1, 14336, 4096), (12, 14336, 4096), (1, 14331, 4096), (16, 14352, 4096),
                                   (7, 14496, 2048)])
def test_htile_decode_shared_tail_vs_oracle(M, N, K):
    """Row-owned decode whose 16-row tiles leave a remainder over the SMs (on 148
    SMs: 8 or 9 leftover tiles of 256-k units shared by up to 144 CTAs, a ragged
    last tile at N = 14331): the leftover rows within 1e-5 (precise) and 1e-2 (fast)
    of the oracle on their own, the whole y too, BF16 y, and bit-identical repeated
    calls (the shared units are added in unit order, whatever CTA finishes last)."""
    from glint_b200 import glint_cuda
    L = glint_cuda.load()
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    tiles = (N + 15) // 16
    row0 = 16 * (tiles // sms) * sms  # first shared row when the tail split applies
    bits = synth_bf16(N * K, seed=N * 3 + M)
    ho, po, ao = O.encode_bf16(bits, 64)
    x = O.f32_to_bf16(np.random.default_rng(M * K + 1).normal(0, 1, M * K).astype(np.float32))
    ref = O.htile(ho, po, ao, x, M, N, K, 64).astype(np.float64)
    dev = [torch.from_numpy(a).cuda() for a in (ho, po, ao)]
    dx = to_dev_bf16(x).view(M, K)
    for _ in range(2):  # the unit counters are zero again after each call
        yp = D().htile(dx, *dev, N, 64, mode="precise")
        yp2 = D().htile(dx, *dev, N, 64, mode="precise")
        yf = D().htile(dx, *dev, N, 64, mode="fast")
        yb = D().htile(dx, *dev, N, 64, mode="fast", out_dtype=torch.bfloat16)
        torch.cuda.synchronize()
        assert L.glint_kernel_error(1) == 0
        assert torch.equal(yp, yp2)
        p, f, b = yp.cpu().numpy(), yf.cpu().numpy(), yb.float().cpu().numpy()
        assert rel_err(p[:, row0:], ref[:, row0:]) <= PRECISE_TOL, rel_err(p[:, row0:], ref[:, row0:])
        assert rel_err(f[:, row0:], ref[:, row0:]) <= FAST_TOL
        assert rel_err(p, ref) <= PRECISE_TOL
        assert rel_err(f, ref) <= FAST_TOL
        assert rel_err(b, ref) <= FAST_TOL
