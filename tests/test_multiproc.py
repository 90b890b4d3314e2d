"""Multi-rank host logic on CPU with the gloo backend (world_size 2).

The column-parallel linear (glint_b200/tp.py) and the LPT placement of a
conversion job (glint_b200/shard.py) are exercised with real process groups; the
per-rank compute is the oracle (tests only), so the gathered results must equal a
single-process oracle run bit for bit.  The NCCL variant of the column-parallel
test needs two GPUs and is marked `gpu`.
"""
import os
import socket
import sys
import tempfile
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

ROOT = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _init(rank, world, port, backend="gloo"):
    import datetime
    import torch.distributed as dist
    sys.path.insert(0, str(ROOT))
    sys.path.insert(0, str(ROOT / "oracle"))
    dist.init_process_group(backend, init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world,
                            timeout=datetime.timedelta(seconds=60))
    return dist


def _weights(N, K, seed):
    import glint_oracle as O
    rng = np.random.default_rng(seed)
    w = rng.normal(0, 0.02, N * K).astype(np.float32)
    w[rng.choice(N * K, size=max(1, N * K // 1000), replace=False)] *= np.float32(20)
    return O.f32_to_bf16(w)


def _column_parallel_worker(rank, world, port, N, K, M):
    dist = _init(rank, world, port)
    import glint_oracle as O
    from glint_b200 import tp
    bits = _weights(N, K, 11)
    hole, plug, am = O.encode_bf16(bits, 64)
    x = O.f32_to_bf16(np.random.default_rng(5).normal(0, 1, M * K).astype(np.float32))
    sh = tp.ColumnShard.from_full(torch.from_numpy(hole), torch.from_numpy(plug), torch.from_numpy(am),
                                  N, K, 64, rank, world)

    def local(xx, s):  # the oracle stands in for the rank's kernel
        return torch.from_numpy(O.htile(s.hole.numpy(), s.plug.numpy(), s.absmax.numpy(), xx, M, s.rows, K, 64))

    y = tp.column_parallel(x, sh, world, rank, local_fn=local)
    ref = O.htile(hole, plug, am, x, M, N, K, 64)
    assert y.shape == (M, N)
    assert np.array_equal(y.numpy(), ref), "gathered columns differ from the single-rank result"
    dist.destroy_process_group()


@pytest.mark.parametrize("N,K,M", [(200, 256, 3), (256, 128, 1), (48, 64, 5)])
def test_column_parallel_gloo(N, K, M):
    """Uneven and even row splits (16-row boundaries) reassemble y exactly."""
    mp.spawn(_column_parallel_worker, args=(2, _free_port(), N, K, M), nprocs=2, join=True)


def _lpt_worker(rank, world, port, outdir):
    dist = _init(rank, world, port)
    import glint_oracle as O
    from glint_b200 import shard
    shapes = [(64, 64), (130, 64), (17, 33), (256, 32), (3, 5), (96, 128), (1, 1)]
    plan = shard.lpt_assign([r * c for r, c in shapes], world)
    mine = {}
    for i in plan[rank]:
        r, c = shapes[i]
        h, p, a = O.encode_bf16(_weights(r, c, 100 + i), 64)
        mine[i] = (h.tobytes(), p.tobytes(), a.tobytes())
    gathered = [None] * world
    dist.all_gather_object(gathered, mine)
    if rank == 0:
        merged = {}
        for d in gathered:
            assert not set(d) & set(merged), "a tensor was encoded by two ranks"
            merged.update(d)
        assert sorted(merged) == list(range(len(shapes))), "a tensor was not encoded"
        for i, (r, c) in enumerate(shapes):
            h, p, a = O.encode_bf16(_weights(r, c, 100 + i), 64)
            assert merged[i] == (h.tobytes(), p.tobytes(), a.tobytes())
        Path(outdir, "ok").write_text("1")
    dist.destroy_process_group()


def test_lpt_sharded_encode_gloo():
    """Per-tensor placement over two ranks: every tensor once, bytes identical to one rank."""
    with tempfile.TemporaryDirectory() as d:
        mp.spawn(_lpt_worker, args=(2, _free_port(), d), nprocs=2, join=True)
        assert Path(d, "ok").read_text() == "1"


def _nccl_worker(rank, world, port, N, K, M):
    torch.cuda.set_device(rank)
    dist = _init(rank, world, port, backend="nccl")
    import glint_oracle as O
    from glint_b200 import device as D
    from glint_b200 import tp
    bits = _weights(N, K, 21)
    hole, plug, am = (torch.from_numpy(a).cuda() for a in O.encode_bf16(bits, 64))
    xb = O.f32_to_bf16(np.random.default_rng(6).normal(0, 1, M * K).astype(np.float32))
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16).view(M, K)
    sh = tp.ColumnShard.from_full(hole, plug, am, N, K, 64, rank, world)
    y = tp.column_parallel(x, sh, world, rank, mode="precise")
    full = D.htile(x, hole, plug, am, N, 64, mode="precise")
    torch.cuda.synchronize()
    ref = O.htile(*(t.cpu().numpy() for t in (hole, plug, am)), xb, M, N, K, 64).astype(np.float64)
    # a rank's split of K differs from the one-GPU split, so compare within the precise bound
    for got in (y, full):
        err = np.abs(got.cpu().numpy().astype(np.float64) - ref).max() / max(1.0, np.abs(ref).max())
        assert err <= 1e-5, err
    dist.destroy_process_group()


@pytest.mark.gpu
def test_column_parallel_nccl_two_gpus():
    """The same reassembly over NCCL with the CUDA kernel on each of two GPUs
    (precise mode, against the oracle)."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_nccl_worker, args=(2, _free_port(), 4096, 4096, 4), nprocs=2, join=True)


def _gather_worker(rank, world, port):
    import os
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist = _init(rank, world, port, backend="nccl")
    from glint_b200 import device as D
    from glint_b200 import glint_cuda
    from glint_b200 import tp
    L = glint_cuda.load()
    L.glint_kernel_error(1)
    g = torch.Generator(device="cuda")
    g.manual_seed(31)  # the same weights and activations on every rank
    # 4096 rows per rank run the row-owned decode, 1024 the stream-K decode
    for N, K in [(8192, 4096), (2048, 4096)]:
        w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        hole, plug, am = D.encode(w, 64)
        sh = tp.ColumnShard.from_full(hole, plug, am, N, K, 64, rank, world)
        for M, dt, mode, tol in [(1, torch.float32, "precise", 1e-5), (4, torch.bfloat16, "fast", 1e-2),
                                 (16, torch.float32, "fast", 1e-2), (32, torch.float32, "fast", 1e-2),
                                 (32, torch.float32, "precise", 1e-5)]:
            pg = tp.PeerGather({"y": (M, N, dt)}, world, rank)
            for _ in range(3):  # consecutive calls alternate the buffers and reuse the counters
                x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
                y = pg.linear(x, sh, "y", mode=mode)
                ref = D.htile(x, hole, plug, am, N, 64, mode=mode, out_dtype=dt)
                torch.cuda.synchronize()
                err = float((y.float() - ref.float()).abs().max() / max(1.0, float(ref.float().abs().max())))
                assert err <= tol, (N, M, mode, err)
            pg.close()
    assert L.glint_kernel_error(1) == 0
    N, K = sh.N, sh.K
    # a rank that skips a gathered call: the other's kernel gives up after about a
    # second with the error word set, instead of hanging
    pg = tp.PeerGather({"y": (1, N, torch.float32)}, world, rank)
    if rank == 0:
        x = torch.randn((1, K), generator=g, device="cuda").to(torch.bfloat16)
        pg.linear(x, sh, "y")
        torch.cuda.synchronize()
        assert L.glint_kernel_error(1) == 1
    pg.close()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_gathered_decode_two_gpus():
    """Column-parallel decode with the all-gather fused into the kernel (peer
    stores over NVLink, CUDA IPC buffers): every rank ends with the whole y, equal
    to the one-GPU decode within the precise / fast bounds, over repeated calls."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_gather_worker, args=(2, _free_port()), nprocs=2, join=True)


def _prefill_gather_worker(rank, world, port):
    import os
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist = _init(rank, world, port, backend="nccl")
    from glint_b200 import device as D
    from glint_b200 import glint_cuda
    from glint_b200 import tp
    L = glint_cuda.load()
    L.glint_kernel_error(1)
    g = torch.Generator(device="cuda")
    g.manual_seed(47)  # the same weights and activations on every rank
    # (N, K, M): 7168 rows per rank at M = 2048 give 224 tiles on the CTA pairs, so
    # the stream-K remainder (split tiles summed by their last contributor) runs
    # gathered too; M = 320 leaves the second activation tile a quarter full
    for N, K, M, dt in [(14336, 4096, 2048, torch.float32), (8192, 4096, 320, torch.bfloat16)]:
        w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
        hole, plug, am = D.encode(w, 64)
        del w
        sh = tp.ColumnShard.from_full(hole, plug, am, N, K, 64, rank, world)
        assert tp.PeerGather.supported(M, sh.rows, "fast") and not tp.PeerGather.supported(M, sh.rows, "precise")
        pg = tp.PeerGather({"y": (M, N, dt)}, world, rank)
        for _ in range(3):  # consecutive calls alternate the buffers and reuse the counters
            x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
            y = pg.linear(x, sh, "y", mode="fast")
            mine = D.htile(x, sh.hole, sh.plug, sh.absmax, sh.rows, 64, mode="fast", out_dtype=dt)
            full = D.htile(x, hole, plug, am, N, 64, mode="fast", out_dtype=dt)
            torch.cuda.synchronize()
            # this rank's columns: the same kernel on the same shard, bit for bit
            assert torch.equal(y[:, sh.n0:sh.n0 + sh.rows], mine), (N, M)
            # every column: the one-GPU GEMM's bound
            err = float((y.float() - full.float()).abs().max() / max(1.0, float(full.float().abs().max())))
            assert err <= 1e-2, (N, M, err)
            # every rank holds the same y
            sums = [torch.zeros(2, dtype=torch.float64, device="cuda") for _ in range(world)]
            dist.all_gather(sums, torch.stack([y.double().sum(), y.double().abs().sum()]))
            assert all(torch.equal(sums[0], t) for t in sums), (N, M)
        pg.close()
        del hole, plug, am, sh
    # a column shard gathered on its own (glint_gather_stream): BF16 from a strided view
    # and f32, repeated, every rank ends with the whole [M, N]
    from glint_b200 import shard as SH
    for dt, M, N in [(torch.bfloat16, 4, 8192), (torch.float32, 32, 1024)]:
        full = torch.randn((M, N), generator=g, device="cuda").to(dt)  # the same on every rank
        n0, n1 = SH.column_shard(N, world, rank)
        pg = tp.PeerGather({"a": (M, N, dt)}, world, rank)
        for _ in range(3):
            got = pg.gather(full[:, n0:n1], "a", n0)
            torch.cuda.synchronize()
            assert torch.equal(got, full), (dt, M, N)
            full = full * 2
        pg.close()
    assert L.glint_kernel_error(1) == 0
    # a rank that skips a gathered prefill call: the other's GEMM gives up after
    # about a second with the error word set, instead of hanging
    N, K, M = 4096, 1024, 128
    w = (torch.randn(N * K, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    hole, plug, am = D.encode(w, 64)
    sh = tp.ColumnShard.from_full(hole, plug, am, N, K, 64, rank, world)
    pg = tp.PeerGather({"y": (M, N, torch.float32)}, world, rank)
    if rank == 0:
        x = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
        pg.linear(x, sh, "y", mode="fast")
        torch.cuda.synchronize()
        assert L.glint_kernel_error(1) == 1
    pg.close()
    dist.destroy_process_group()


@pytest.mark.gpu
def test_gathered_prefill_two_gpus():
    """Column-parallel prefill with the all-gather fused into the tcgen05 GEMM's
    epilogue: every rank ends with the whole y; its own columns equal the
    ungathered GEMM on its shard bit for bit and every column is within the fast
    bound of the one-GPU GEMM, over repeated calls (data-parallel and stream-K
    tiles, ragged M, f32 and BF16 y); a skipped call times out with an error."""
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    mp.spawn(_prefill_gather_worker, args=(2, _free_port()), nprocs=2, join=True)
