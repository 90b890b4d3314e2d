"""Column-parallel GLINT linears across ranks (one process per GPU).

The reference has no multi-GPU code; its H-TILE contract (cuda/glint_htile.cu:124-164)
is one device computing y[M, N] = x[M, K] . W[N, K]^T from the packed planes.  Over P
ranks the weight shards column-parallel: rank r holds packed rows [n0, n1) of W
(`shard.column_shard`, boundaries on 16-row multiples), which for K % blocksize == 0
is one contiguous byte range of hole and plug and one float range of absmax
(`shard.shard_planes`).  Each rank runs its local H-TILE kernel on its rows and a
single all-gather (NCCL over NVLink/NVSwitch on a B200 node) reassembles y where the
consumer needs whole rows.  Activations are replicated, so there is no other
exchange; nothing reads another GPU's memory directly.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Callable, Optional

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
