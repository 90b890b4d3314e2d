"""GPU parity of the K-major decode (glint_b200/csrc/kmajor.cu, include/glint_km.h)
through its C ABI, against the CPU oracle (oracle/glint_oracle.c restating the
reference's Mojo decoders, pinned in tests/test_kmajor_oracle.py).

Bars: layout bytes and the selected channel list bit-exact; the parent GEMV and
the correction within 1e-5 * max(1, max|y|) of an f64 sum (they sum in a fixed
order of their own, not the reference's sequential one); with every channel
selected, the decode step within the same bound of the precise H-TILE.
"""
import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import glint_oracle as O  # noqa: E402

TOL = 1e-5
SHAPES = [(14336, 4096), (4096, 14336), (1024, 64), (8, 64), (264, 192), (2048, 8192)]


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


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def _weight(n, K, seed):
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, n * K).astype(np.float32)
    w[rng.choice(n * K, size=max(1, n * K // 1000), replace=False)] *= np.float32(20)
    bits = O.f32_to_bf16(w)
    h, p, a = D().encode(_bf16(bits), 64)
    return h, p, a


def _x(K, seed):
    return O.f32_to_bf16(np.random.default_rng(seed).normal(0, 1, K).astype(np.float32))


def _err(y, ref):
    return float(np.abs(np.asarray(y, np.float64) - ref).max() / max(1.0, float(np.abs(ref).max())))


def _parent_f64(hk, sk, x, n, K):
    """sum_c PARENT[h] * scale * x[c] in f64 from the K-major planes"""
    nib = np.stack([hk & 15, hk >> 4], axis=1).reshape(K, n)
    parent = np.asarray(_PARENT, np.float64)[nib]
    s = np.repeat(sk.reshape(K // 64, n), 64, axis=0).astype(np.float64)
    return (parent * s * O.bf16_to_f32(x).astype(np.float64)[:, None]).sum(axis=0)


_PARENT = None


@pytest.fixture(scope="module", autouse=True)
def parent_table():
    global _PARENT
    import re
    from pathlib import Path
    txt = (Path(__file__).resolve().parents[1] / "include" / "glint_cells.h").read_text()
    line = txt.split("#define GLINT_PARENT_INIT")[1].split("\n")[0]
    _PARENT = np.array([float.fromhex(v[:-1]) for v in re.findall(r"-?0x[0-9a-f.]+p[-+][0-9]+f", line)], np.float32)


@pytest.mark.parametrize("n,K", SHAPES)
def test_layout_bytes_equal_oracle(n, K):
    h, p, a = _weight(n, K, n + K)
    hk, pk, sk = D().to_kmajor(h, p, a, n, K)
    ohk, opk, osk = O.to_kmajor(h.cpu().numpy(), p.cpu().numpy(), a.cpu().numpy(), n, K)
    torch.cuda.synchronize()
    assert np.array_equal(hk.cpu().numpy(), ohk)
    assert np.array_equal(pk.cpu().numpy(), opk)
    assert np.array_equal(sk.cpu().numpy().view(np.uint32), osk.view(np.uint32))


@pytest.mark.parametrize("n,K", SHAPES)
def test_parent_gemv(n, K):
    h, p, a = _weight(n, K, 3 * n + K)
    hk, pk, sk = D().to_kmajor(h, p, a, n, K)
    x = _x(K, 5)
    y = D().gemv_km(_bf16(x), hk, sk, n)
    ref = _parent_f64(hk.cpu().numpy(), sk.cpu().numpy(), x, n, K)
    assert _err(y.cpu().numpy(), ref) <= TOL, (n, K)
    # and the oracle's restatement of the reference's own order agrees as well
    assert _err(O.gemv_km(hk.cpu().numpy(), sk.cpu().numpy(), x, n, K), ref) <= TOL


def test_select_bit_exact():
    rng = np.random.default_rng(1)
    for K in (64, 192, 4096, 14336, 28672, 65536):
        x = _x(K, K)
        # plant ties, zeros of both signs, infinities and a NaN
        x[rng.choice(K, 8, replace=False)] = x[0]
        x[1:3] = [0x0000, 0x8000]
        if K > 8:
            x[5:8] = [0x7F80, 0xFF80, 0x7FC0]
        xd = _bf16(x)
        for nsel in sorted({0, 1, 2, 7, K // 10, K // 2, K - 1, K, K + 3}):
            idx, cnt = D().select_topk(xd, nsel)
            want = O.select_topk(x, nsel)
            c = int(cnt.item())
            assert c == len(want), (K, nsel)
            assert np.array_equal(idx[:c].cpu().numpy(), want), (K, nsel)


@pytest.mark.parametrize("n,K,pct", [(14336, 4096, 10), (4096, 14336, 3), (1024, 64, 50), (264, 192, 100)])
@pytest.mark.parametrize("host_plug", [False, True])
def test_correction(n, K, pct, host_plug):
    h, p, a = _weight(n, K, 7 * n + K)
    plug_host = torch.empty(K * n // 2, dtype=torch.uint8).pin_memory() if host_plug else None
    hk, pk, sk = D().to_kmajor(h, p, a, n, K, plug_out=plug_host)
    torch.cuda.synchronize()
    x = _x(K, 11)
    xd = _bf16(x)
    nsel = (pct * K + 99) // 100
    idx, cnt = D().select_topk(xd, nsel)
    y0 = D().gemv_km(xd, hk, sk, n)
    y = D().apply_corr_k(y0.clone(), xd, hk, pk, sk, idx, cnt, n)
    hkn, pkn, skn = hk.cpu().numpy(), pk.cpu().numpy(), sk.cpu().numpy()
    sel = O.select_topk(x, nsel)
    want = O.apply_corr_k(y0.cpu().numpy(), hkn, pkn, skn, x, sel, n, K)
    assert _err(y.cpu().numpy(), want.astype(np.float64)) <= TOL, (n, K, pct, host_plug)
    # the fused step gives the same numbers as the three calls
    ys, idx2, cnt2 = D().gemv_select(xd, hk, pk, sk, n, nsel)
    assert int(cnt2.item()) == len(sel)
    assert torch.equal(ys, y)


@pytest.mark.parametrize("n,K", [(14336, 4096), (4096, 14336), (264, 192)])
def test_full_selection_is_the_glint_gemv(n, K):
    """Every channel selected: parent + correction == the full GLINT GEMV (precise)."""
    h, p, a = _weight(n, K, 13 * n + K)
    hk, pk, sk = D().to_kmajor(h, p, a, n, K)
    x = _x(K, 17)
    xd = _bf16(x)
    y, _, cnt = D().gemv_select(xd, hk, pk, sk, n, K)
    assert int(cnt.item()) == K
    ref = D().htile(xd.view(1, K), h, p, a, n, 64, mode="precise")[0]
    o = O.htile(h.cpu().numpy(), p.cpu().numpy(), a.cpu().numpy(), x, 1, n, K, 64)[0]
    assert _err(y.cpu().numpy(), o.astype(np.float64)) <= TOL
    assert _err(ref.cpu().numpy(), o.astype(np.float64)) <= TOL


def test_repeated_steps_reuse_scratch_and_are_deterministic():
    n, K = 4096, 4096
    h, p, a = _weight(n, K, 99)
    hk, pk, sk = D().to_kmajor(h, p, a, n, K)
    outs = []
    for i in range(4):
        xd = _bf16(_x(K, 40 + (i % 2)))
        y, idx, cnt = D().gemv_select(xd, hk, pk, sk, n, 400)
        outs.append(y.clone())
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[2]) and torch.equal(outs[1], outs[3])
    assert not torch.equal(outs[0], outs[1])


def test_argument_checks():
    L = D().lib()
    n, K = 64, 128
    hk = torch.zeros(K * n // 2, dtype=torch.uint8, device="cuda")
    sk = torch.zeros(K // 64 * n, dtype=torch.float32, device="cuda")
    x = torch.zeros(K, dtype=torch.bfloat16, device="cuda")
    y = torch.zeros(n, dtype=torch.float32, device="cuda")
    s = D()._stream(None)
    assert L.glint_gemv_km_stream(hk.data_ptr(), sk.data_ptr(), x.data_ptr(), y.data_ptr(), 60, K, s) == -1
    assert L.glint_gemv_km_stream(hk.data_ptr(), sk.data_ptr(), x.data_ptr(), y.data_ptr(), n, 100, s) == -1
    assert L.glint_gemv_km_stream(None, sk.data_ptr(), x.data_ptr(), y.data_ptr(), n, K, s) == -1
    assert L.glint_select_topk_stream(x.data_ptr(), K, -1, y.data_ptr(), y.data_ptr(), s) == -1
    assert L.glint_kmajor_from_rowmajor(hk.data_ptr(), hk.data_ptr(), sk.data_ptr(), n, K, 32, hk.data_ptr(),
                                        hk.data_ptr(), sk.data_ptr(), s) == -2
    torch.cuda.synchronize()
