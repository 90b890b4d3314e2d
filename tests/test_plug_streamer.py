"""Plug streamer (include/glint_plug_streamer.h): the reference's own checks
(tests/test_glint_plug_streamer.cu:1-125, tests/test_streamer_real_weights.cu:1-284)
restated over the C ABI.

- Every pass over 1, 2, 3 and 32 layers reads only its own layer's bytes, also
  when each read is delayed by a spin on the compute stream (so a refill that
  skipped its slot wait would land before the read); every layer is copied
  once per pass.
- Call order: release before start/acquire, out-of-order release and acquire,
  double release, and start during a pass return the reference's codes.
- H-TILE fed from the streamer's slots is bit-identical to the same call with
  the plug resident, over plain, poisoned (a released slot is overwritten with
  random bytes) and delayed passes.
"""
import ctypes

import numpy as np
import pytest
import torch

from glint_b200 import glint_cuda


def test_bad_arguments_rejected_without_gpu():
    L = glint_cuda.load()
    assert L is not None
    h = ctypes.c_void_p()
    sizes = (ctypes.c_uint64 * 65)(*([16] * 65))
    assert L.glint_plug_streamer_create(ctypes.byref(h), 0, sizes, None, None) == -1
    assert L.glint_plug_streamer_create(ctypes.byref(h), 65, sizes, None, None) == -1
    assert L.glint_plug_streamer_create(None, 1, sizes, None, None) == -1
    assert L.glint_plug_streamer_create(ctypes.byref(h), 1, None, None, None) == -1
    assert L.glint_plug_streamer_start(None) == -1
    p = ctypes.c_void_p()
    assert L.glint_plug_streamer_acquire(None, 0, ctypes.byref(p)) == -1
    assert L.glint_plug_streamer_release(None, 0) == -1
    assert L.glint_plug_streamer_set_host_data(None, 0, None, 0) == -1
    assert L.glint_plug_streamer_get_stats(None, None) == -1
    assert L.glint_plug_streamer_host_buffer(None, 0) is None
    L.glint_plug_streamer_destroy(None)
    L.glint_plug_streamer_reset_stats(None)


LAYER_BYTES = 4 << 20


def _pattern(layer: int, n: int) -> np.ndarray:
    # tests/test_glint_plug_streamer.cu:30-33: byte i of layer l is (l*37 + i % 251) & 0xFF
    return ((layer * 37 + np.arange(n, dtype=np.int64) % 251) & 0xFF).astype(np.uint8)


def _delay_cycles(ms: float) -> int:
    return int(ms * 1.965e6)  # torch.cuda._sleep counts SM cycles (max SM clock 1965 MHz)


@pytest.mark.gpu
@pytest.mark.parametrize("n_layers", [1, 2, 3, 32])
def test_passes_read_their_own_layer(n_layers):
    from glint_b200.streamer import PlugStreamer, device_bytes
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    expect = [torch.from_numpy(_pattern(l, LAYER_BYTES)).cuda() for l in range(n_layers)]
    torch.cuda.synchronize()
    passes, delay = 3, _delay_cycles(5.0)
    with PlugStreamer([LAYER_BYTES] * n_layers, copy_s.cuda_stream, comp_s.cuda_stream) as s:
        for l in range(n_layers):
            assert s.set_host_data(l, _pattern(l, LAYER_BYTES)) == 0
        bad = torch.zeros((), dtype=torch.int64, device="cuda")
        for _ in range(passes):
            assert s.start() == 0
            for l in range(n_layers):
                rc, ptr = s.acquire(l)
                assert rc == 0 and ptr
                with torch.cuda.stream(comp_s):
                    torch.cuda._sleep(delay)
                    bad += (device_bytes(ptr, LAYER_BYTES) != expect[l]).sum()
                assert s.release(l) == 0
        torch.cuda.synchronize()
        st = s.stats()
        assert int(bad.item()) == 0, "a pass read another layer's bytes"
        assert st["total_h2d_bytes"] == passes * n_layers * LAYER_BYTES
        assert st["n_layers"] == n_layers and len(st["per_layer_stall_ms"]) == n_layers
        assert all(v >= 0.0 for v in st["per_layer_stall_ms"])


@pytest.mark.gpu
def test_call_order_codes():
    """tests/test_glint_plug_streamer.cu:85-106 and test_streamer_real_weights.cu:218-222."""
    from glint_b200.streamer import PlugStreamer
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    with PlugStreamer([1 << 20] * 3, copy_s.cuda_stream, comp_s.cuda_stream) as s:
        for l in range(3):
            assert s.set_host_data(l, _pattern(l, 1 << 20)) == 0
        assert s.set_host_data(0, np.zeros(5, np.uint8)) == -2       # size differs
        assert s.release(0) == -11                                    # before start
        assert s.acquire(0)[0] == -10                                 # before start
        assert s.start() == 0
        assert s.start() == -6                                        # pass in flight
        assert s.release(0) == -11                                    # before acquire(0)
        assert s.acquire(1)[0] == -10                                 # before release(0)
        assert s.acquire(0)[0] == 0
        assert s.release(1) == -11                                    # before release(0)
        assert s.release(0) == 0
        assert s.release(0) == -11                                    # twice
        assert s.release(1) == -11                                    # before acquire(1)
        assert s.acquire(1)[0] == 0 and s.release(1) == 0
        assert s.acquire(2)[0] == 0 and s.release(2) == 0
        assert s.start() == 0                                         # next pass after the last release
        for l in range(3):
            assert s.acquire(l)[0] == 0 and s.release(l) == 0
        torch.cuda.synchronize()


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 4, 130])
def test_streamed_htile_bitwise(M):
    """Plugs through the ring give the same y as resident plugs, bit for bit, over
    plain, poisoned and delayed passes (tests/test_streamer_real_weights.cu:171-260)."""
    from glint_b200 import device as D
    from glint_b200.streamer import PlugStreamer, device_bytes
    g = torch.Generator(device="cuda")
    g.manual_seed(11)
    shapes = [(3072, 1024), (1024, 1024), (8192, 1024), (1024, 4096), (2048, 512)]  # (N, K) per unit
    units = []
    for N, K in shapes:
        w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        hole, plug, am = D.encode(w, 64)
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        units.append((N, K, hole, plug, am, x))
    kinds = ["plain", "plain", "poison", "poison", "delay", "delay"]
    copy_s, comp_s = torch.cuda.Stream(), torch.cuda.Stream()
    copy_s.wait_stream(torch.cuda.current_stream())
    comp_s.wait_stream(torch.cuda.current_stream())
    resident = []
    for N, K, hole, plug, am, x in units:
        for mode in ("fast", "precise"):
            resident.append(D.htile(x, hole, plug, am, N, 64, mode=mode, stream=comp_s))
    sizes = [u[3].numel() for u in units]
    poison = torch.randint(0, 256, (max(sizes),), dtype=torch.uint8, generator=torch.Generator().manual_seed(5)).pin_memory()
    delay = _delay_cycles(5.0)
    outs = []
    with PlugStreamer(sizes, copy_s.cuda_stream, comp_s.cuda_stream) as s:
        for i, u in enumerate(units):
            s.host_buffer(i)[:] = u[3].cpu().numpy()   # write plugs straight into the pinned buffers
        torch.cuda.synchronize()
        for kind in kinds:
            assert s.start() == 0
            if len(units) > 1:
                assert s.acquire(1)[0] == -10
            ys = []
            for i, (N, K, hole, plug, am, x) in enumerate(units):
                rc, ptr = s.acquire(i)
                assert rc == 0 and ptr
                slot = device_bytes(ptr, sizes[i])
                with torch.cuda.stream(comp_s):
                    if kind == "delay":
                        torch.cuda._sleep(delay)
                for mode in ("fast", "precise"):
                    ys.append(D.htile(x, hole, slot, am, N, 64, mode=mode, stream=comp_s))
                assert s.release(i) == 0
                if kind == "poison":
                    ev = torch.cuda.Event()
                    ev.record(comp_s)
                    copy_s.wait_event(ev)
                    with torch.cuda.stream(copy_s):
                        slot.copy_(poison[: sizes[i]], non_blocking=True)
            outs.append(ys)
        torch.cuda.synchronize()
    for p, ys in enumerate(outs):
        for j, (a, b) in enumerate(zip(resident, ys)):
            assert torch.equal(a, b), f"pass {p} ({kinds[p]}), unit {j // 2} mode {('fast', 'precise')[j % 2]} differs"
