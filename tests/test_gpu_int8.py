"""GPU parity of the INT8 W8A8 GEMM and its res4 late plug (glint_b200/csrc/int8_gemm.cu,
include/int8_mma_gemm.h) through the reference's own entry points: the activation
codes and scales and every output bit-exact against the oracle (oracle/glint_oracle.c)
and against the reference's cuda/int8_mma_gemm.cu built unchanged for sm_100a
(oracle/_ref/libp7_int8.so, when staged).  The int32 block sums are exact and the f32
steps are one fixed sequence, so the tiling does not change any bit."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

import glint_oracle as O  # noqa: E402

REF = Path(__file__).resolve().parents[1] / "oracle" / "_ref" / "libp7_int8.so"
# M > 64 with K % 128 == 0 runs the tcgen05 kind::i8 kernel (every entry point and
# pass, the fused plug included); the rest run the mma.sync kernel
SHAPES = [(1, 4096, 4096), (7, 1000, 192), (24, 1000, 640), (64, 128, 64), (130, 300, 640), (32, 4096, 14336),
          (96, 520, 384), (256, 4096, 4096), (520, 1000, 2048)]


@pytest.fixture(scope="module", autouse=True)
def gpu():
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from glint_b200 import build
    build.build()
    O.set_threads()
    torch.cuda.set_device(0)


def I8():
    from glint_b200 import int8
    return int8


def _bf16(bits):
    return torch.from_numpy(bits.astype(np.uint16).view(np.int16)).cuda().view(torch.bfloat16)


def _case(m, n, k, seed):
    rng = np.random.default_rng(seed)
    xb = O.f32_to_bf16(rng.normal(0, 1, m * k).astype(np.float32))
    wq, ws = O.int8_quant(O.f32_to_bf16(rng.normal(0, 0.02, n * k).astype(np.float32)), n, k)
    q4 = rng.integers(0, 256, n * k // 2, dtype=np.uint8)
    ps = (rng.random(n * (k // 64)) * 2e-5).astype(np.float32)
    return xb, wq, ws, q4, ps


def _dev(xb, wq, ws, q4, ps, m, k):
    return (_bf16(xb).view(m, k), torch.from_numpy(wq).cuda().view(-1, k), torch.from_numpy(ws).cuda(),
            torch.from_numpy(q4).cuda(), torch.from_numpy(ps).cuda())


def _oracle_all(xb, wq, ws, q4, ps, m, n, k):
    xq, sx = O.int8_quant(xb, m, k)
    rq, sr = O.int8_quant(xb, m, k, prev=(xq, sx))
    nib = (np.stack([q4 & 15, q4 >> 4], axis=1).reshape(-1).astype(np.int16) - 8).astype(np.int8)
    base = O.int8_gemm(xq, sx, wq, ws, m, n, k)
    plug = O.int8_gemm(xq, sx, nib, ps, m, n, k, y=base, accumulate=True)
    fused = O.int8_gemm(xq, sx, wq, ws, m, n, k, plug=(q4, ps))
    res = O.int8_gemm(rq, sr, wq, ws, m, n, k, y=base, accumulate=True)
    resp = O.int8_gemm(rq, sr, nib, ps, m, n, k,
                       y=O.int8_gemm(xq, sx, nib, ps, m, n, k, y=res, accumulate=True), accumulate=True)
    return {"gemm": base, "plug": plug, "fused": fused, "resolve": res, "resolve_plug": resp}, (xq, sx, rq, sr)


def _run(lib, d, kind, plug):
    x, wq, ws, q4, ps = d
    y, sc = I8().gemm(x, wq, ws, plug=(q4, ps) if plug else None, kind=kind, lib=lib)
    torch.cuda.synchronize()
    return y.cpu().numpy(), sc


@pytest.mark.parametrize("m,n,k", [s for s in SHAPES if s[0] * s[1] * s[2] <= 1 << 26])
def test_int8_bit_exact_against_oracle(m, n, k):
    xb, wq, ws, q4, ps = _case(m, n, k, m + n + k)
    want, (xq, sx, rq, sr) = _oracle_all(xb, wq, ws, q4, ps, m, n, k)
    d = _dev(xb, wq, ws, q4, ps, m, k)
    for kind, plug, key in [("gemm", False, "gemm"), ("plug", True, "plug"), ("fused", True, "fused"),
                            ("resolve", False, "resolve"), ("resolve", True, "resolve_plug")]:
        y, sc = _run(None, d, kind, plug)
        assert np.array_equal(sc["xq"].cpu().numpy(), xq) and np.array_equal(sc["sx"].cpu().numpy(), sx)
        if kind == "resolve":
            assert np.array_equal(sc["rq"].cpu().numpy(), rq) and np.array_equal(sc["sr"].cpu().numpy(), sr)
        assert np.array_equal(y.view(np.uint32), want[key].view(np.uint32)), (kind, plug)


@pytest.mark.skipif(not REF.is_file(), reason="the reference's INT8 kernel is not staged in oracle/_ref")
@pytest.mark.parametrize("m,n,k", SHAPES)
def test_int8_bit_exact_against_the_reference_kernel(m, n, k):
    ref = I8().bind(ctypes.CDLL(str(REF)))
    xb, wq, ws, q4, ps = _case(m, n, k, 3 * m + n + k)
    d = _dev(xb, wq, ws, q4, ps, m, k)
    for kind, plug in [("gemm", False), ("plug", True), ("fused", True), ("resolve", False), ("resolve", True)]:
        mine, _ = _run(None, d, kind, plug)
        theirs, _ = _run(ref, d, kind, plug)
        assert np.array_equal(mine.view(np.uint32), theirs.view(np.uint32)), (m, n, k, kind, plug)


def test_plug_scratch_contents_do_not_matter():
    m, n, k = 16, 512, 256
    xb, wq, ws, q4, ps = _case(m, n, k, 11)
    d = _dev(xb, wq, ws, q4, ps, m, k)
    outs = []
    for fill in (0x55, 0x7F):
        sc = {"plug_i8": torch.full((n * k,), fill, dtype=torch.int8, device="cuda").view(torch.int8)}
        y, _ = I8().gemm(d[0], d[1], d[2], plug=(d[3], d[4]), kind="plug", scratch=sc)
        torch.cuda.synchronize()
        outs.append(y.clone())
    assert torch.equal(outs[0], outs[1])


def test_argument_checks():
    L = I8()._ours()
    lin = I8().Int8MmaLinear(0, 0, 8, 100)
    x = torch.zeros((2, 128), dtype=torch.bfloat16, device="cuda")
    assert L.int8_mma_gemm(x.data_ptr(), lin, x.data_ptr(), 2, x.data_ptr(), x.data_ptr(), None) != 0
    q = torch.zeros((8, 100), dtype=torch.int8, device="cuda")
    lin = I8().Int8MmaLinear(q.data_ptr(), q.data_ptr(), 8, 100)  # k_in % 64 != 0
    assert L.int8_mma_gemm(x.data_ptr(), lin, x.data_ptr(), 2, x.data_ptr(), x.data_ptr(), None) != 0
