"""Column-parallel GLINT linears across ranks (one process per GPU).

The reference has no multi-GPU code; its H-TILE contract (cuda/glint_htile.cu:124-164)
is one device computing y[M, N] = x[M, K] . W[N, K]^T from the packed planes.  Over P
ranks the weight shards column-parallel: rank r holds packed rows [n0, n1) of W
(`shard.column_shard`, boundaries on 16-row multiples), which for K % blocksize == 0
is one contiguous byte range of hole and plug and one float range of absmax
(`shard.shard_planes`).  Each rank runs its local H-TILE kernel on its rows and a
single all-gather reassembles y where the consumer needs whole rows: either NCCL
(`gather_columns`) or, for decode shapes, fused into the kernel (`PeerGather`: each
rank's kernel stores its rows into every rank's output over NVLink and counts itself
in).  Activations are replicated, so there is no other exchange; no kernel reads
another GPU's memory.
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Dict, Optional, Tuple

import torch

from . import shard


@dataclass
class ColumnShard:
    """This rank's rows [n0, n1) of a GLINT-packed [N, K] weight."""
    n0: int
    n1: int
    N: int
    K: int
    blocksize: int
    hole: torch.Tensor
    plug: torch.Tensor
    absmax: torch.Tensor

    @property
    def rows(self) -> int:
        return self.n1 - self.n0

    @classmethod
    def from_full(cls, hole: torch.Tensor, plug: torch.Tensor, absmax: torch.Tensor, N: int, K: int,
                  blocksize: int, rank: int, world: int, align: int = 16) -> "ColumnShard":
        """Slice rank `rank`'s rows out of whole-weight planes (views, no copy)."""
        if K % blocksize:
            raise ValueError("column-parallel sharding needs K % blocksize == 0")
        n0, n1 = shard.column_shard(N, world, rank, align)
        r = shard.shard_planes((n0, n1), K, blocksize)
        (p0, p1), (a0, a1) = r["planes"], r["absmax"]
        return cls(n0, n1, N, K, blocksize, hole[p0:p1], plug[p0:p1], absmax[a0:a1])


def shard_rows(N: int, world: int, align: int = 16):
    """Row ranges of every rank, in rank order."""
    return [shard.column_shard(N, world, r, align) for r in range(world)]


def gather_columns(y_local: torch.Tensor, N: int, world: int, rank: int, align: int = 16,
                   group=None) -> torch.Tensor:
    """All-gather the ranks' [M, rows_r] output shards into y [M, N].

    Shards are padded to the largest rank's row count so that one
    all_gather_into_tensor moves them all; each rank then keeps the valid
    columns of every shard in rank order."""
    if world == 1:
        return y_local
    import torch.distributed as dist
    ranges = shard_rows(N, world, align)
    width = max(n1 - n0 for n0, n1 in ranges)
    M = y_local.shape[0]
    send = y_local
    if y_local.shape[1] != width:
        send = torch.zeros((M, width), dtype=y_local.dtype, device=y_local.device)
        send[:, : y_local.shape[1]] = y_local
    recv = torch.empty((world * M, width), dtype=y_local.dtype, device=y_local.device)
    dist.all_gather_into_tensor(recv, send.contiguous(), group=group)
    parts = recv.view(world, M, width)
    return torch.cat([parts[r, :, : n1 - n0] for r, (n0, n1) in enumerate(ranges)], dim=1)


class PeerGather:
    """Output buffers shared by the ranks of a group, for column-parallel linears
    whose all-gather is fused into the decode kernel (glint_htile_gather_stream).

    Every rank allocates each named output y[M, N] (and a pair of arrival
    counters) with glint_device_alloc, the CUDA IPC handles are exchanged once over
    the process group, and every rank maps every other rank's buffers.  A gathered
    call computes this rank's rows and stores them into all ranks' y over NVLink;
    when it completes on the stream, the local y holds every rank's rows, with no
    NCCL call and no copy.  All ranks must make the same gathered calls in the
    same order; a rank that skips one makes the others give up after about a
    second with glint_kernel_error() set.  A gathered call may be captured in a
    CUDA graph and replayed (the completion count needs no call number).  Each output has two buffers used in turn, so a
    result stays valid until the second-next call with that name: a rank can only
    start that call once every rank has started the next one, which each rank
    enqueues after its reads of this result.  No multicast objects are created."""

    def __init__(self, outputs: Dict[str, Tuple[int, int, torch.dtype]], world: int, rank: int, group=None):
        from . import glint_cuda
        from .streamer import device_bytes
        self._lib = glint_cuda._require()
        self.world, self.rank = world, rank
        self._local, self._opened = [], []
        self.y: Dict[str, list] = {}
        self._yptrs: Dict[str, list] = {}
        self._calls: Dict[str, int] = {}
        self.shapes = dict(outputs)
        try:
            self._setup(outputs, group, device_bytes)
        except Exception:
            self._release()
            raise

    def _setup(self, outputs, group, device_bytes) -> None:
        import torch.distributed as dist
        lib, world, rank = self._lib, self.world, self.rank

        def alloc(nbytes):
            p = ctypes.c_void_p()
            rc = lib.glint_device_alloc(nbytes, ctypes.byref(p))
            if rc != 0:
                raise RuntimeError(f"glint_device_alloc rc={rc}")
            self._local.append(p.value)
            h = ctypes.create_string_buffer(64)
            rc = lib.glint_ipc_handle(p, h)
            if rc != 0:
                raise RuntimeError(f"glint_ipc_handle rc={rc}")
            return p.value, h.raw

        keys = [(nm, b) for nm in sorted(outputs) for b in (0, 1)]
        mine = {}
        for nm, b in keys:
            M, N, dt = outputs[nm]
            esz = torch.empty((), dtype=dt).element_size()
            ptr, h = alloc(M * N * esz)
            mine[f"{nm}/{b}"] = (ptr, h)
            self.y.setdefault(nm, []).append(device_bytes(ptr, M * N * esz).view(dt).view(M, N))
        fptr, fh = alloc(256)
        mine["__flags__"] = (fptr, fh)
        every = [None] * world
        dist.all_gather_object(every, {k: v[1] for k, v in mine.items()}, group=group)

        def mapped(key):
            arr = (ctypes.c_void_p * world)()
            for r in range(world):
                if r == rank:
                    arr[r] = mine[key][0]
                    continue
                p = ctypes.c_void_p()
                rc = lib.glint_ipc_open(every[r][key], ctypes.byref(p))
                if rc != 0:
                    raise RuntimeError(f"glint_ipc_open rc={rc} (rank {r}, {key})")
                self._opened.append(p.value)
                arr[r] = p.value
            return arr

        for nm, b in keys:
            self._yptrs.setdefault(nm, []).append(mapped(f"{nm}/{b}"))
            self._calls[nm] = 0
        self._flags = mapped("__flags__")
        torch.cuda.synchronize()
        dist.barrier(group=group)

    @staticmethod
    def supported(M: int, rows: int, mode: str = "fast") -> bool:
        """Shapes a gathered call covers, given bs == 64, K % 256 == 0 and 16-byte
        aligned operands: the decode kernels at M <= 32 (both modes) and the
        tcgen05 prefill GEMM at M >= 128 (fast mode)."""
        if rows < 1:
            return False
        return 1 <= M <= 32 or (M >= 128 and mode == "fast")

    def linear(self, x: torch.Tensor, sh: ColumnShard, name: str, mode: str = "fast", stream=None) -> torch.Tensor:
        """y[M, N] = x . W^T on every rank: this rank's rows [n0, n1) computed here,
        the others' written by their ranks.  Returns one of the name's two shared
        local buffers (valid once the call completes on the stream, until the
        second-next call with the same name)."""
        M, N, dt = self.shapes[name]
        if x.shape[0] != M or sh.N != N:
            raise ValueError("output shape differs from the buffer's")
        if not x.is_cuda or x.dtype != torch.bfloat16 or x.dim() != 2 or x.shape[1] != sh.K or not x.is_contiguous():
            raise ValueError("x must be a contiguous bfloat16 CUDA tensor [M, K]")
        if sh.rows < 1:
            # every rank signals every gathered call; a rank without rows cannot, and its
            # peers would give up after about a second
            raise ValueError("a gathered call needs at least one row on every rank (N >= 16 x world)")
        buf = self._calls[name] & 1
        ydt = 1 if dt == torch.bfloat16 else 0
        s = stream if stream is not None else torch.cuda.current_stream()
        rc = self._lib.glint_htile_gather_stream(
            sh.hole.data_ptr(), sh.plug.data_ptr(), sh.absmax.data_ptr(), x.data_ptr(), self._yptrs[name][buf],
            self._flags, self.world, self.rank, ydt, M, sh.rows, sh.K, N, sh.n0, sh.blocksize,
            1 if mode == "fast" else 0, ctypes.c_void_p(s.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"glint_htile_gather_stream rc={rc}")
        self._calls[name] += 1
        return self.y[name][buf]

    def gather(self, shard: torch.Tensor, name: str, n0: int, stream=None) -> torch.Tensor:
        """Columns [n0, n0 + cols) of the named output from this rank's shard
        [M, cols] (any row stride; the output's dtype, BF16 or f32), stored into every
        rank's buffer over NVLink (glint_gather_stream).  Returns one of the name's two
        shared local buffers, whole once the call completes on the stream; the same
        rules as linear() (every rank gathers, in the same order)."""
        M, N, dt = self.shapes[name]
        if shard.dtype != dt or shard.dim() != 2 or shard.shape[0] != M or not shard.is_cuda:
            raise ValueError("shard must be a CUDA [M, cols] tensor of the output's dtype")
        if shard.stride(1) != 1 or n0 < 0 or n0 + shard.shape[1] > N:
            raise ValueError("shard rows must be contiguous and fit the output's columns")
        buf = self._calls[name] & 1
        s = stream if stream is not None else torch.cuda.current_stream()
        rc = self._lib.glint_gather_stream(shard.data_ptr(), shard.element_size(), M, shard.shape[1],
                                           shard.stride(0), self._yptrs[name][buf], self._flags, self.world,
                                           self.rank, N, n0, ctypes.c_void_p(s.cuda_stream))
        if rc != 0:
            raise RuntimeError(f"glint_gather_stream rc={rc}")
        self._calls[name] += 1
        return self.y[name][buf]

    def close(self, group=None) -> None:
        """Unmap the peers' buffers and free this rank's (after every rank is done with them)."""
        import torch.distributed as dist
        if not self._local:
            return
        torch.cuda.synchronize()
        dist.barrier(group=group)
        for p in self._opened:
            self._lib.glint_ipc_close(ctypes.c_void_p(p))
        self._opened = []
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self._release()

    def _release(self) -> None:
        """Unmap and free without synchronising with the other ranks (set-up failure)."""
        for p in self._opened:
            self._lib.glint_ipc_close(ctypes.c_void_p(p))
        for p in self._local:
            self._lib.glint_device_free(ctypes.c_void_p(p))
        self._local, self._opened, self.y = [], [], {}


def column_parallel(x: torch.Tensor, sh: ColumnShard, world: int, rank: int, mode: str = "fast",
                    out_dtype: torch.dtype = torch.float32, group=None, gather: bool = True,
                    local_fn: Optional[Callable[[torch.Tensor, ColumnShard], torch.Tensor]] = None) -> torch.Tensor:
    """y = x . W^T for a column-sharded GLINT weight: the local H-TILE on this
    rank's rows, then (if `gather`) the all-gather.  `local_fn` replaces the local
    kernel call (the CPU tests plug the oracle in); by default it is the CUDA
    kernel, which raises for tensors that are not on a GPU."""
    if local_fn is None:
        from . import device as D
        y_local = D.htile(x, sh.hole, sh.plug, sh.absmax, sh.rows, sh.blocksize, mode=mode, out_dtype=out_dtype)
    else:
        y_local = local_fn(x, sh)
    return gather_columns(y_local, sh.N, world, rank, group=group) if gather else y_local
