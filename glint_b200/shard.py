"""Multi-GPU placement for the GLINT hot path.

Encode and expand are independent per tensor (reference glint_pin.py:133-164
walks them one after another on one device), so a conversion job is split across
ranks with no collective: tensors are assigned by longest-processing-time-first
(LPT) on their weight counts.  Linear layers shard column-parallel over N: rank r
holds packed rows [r*N/P, (r+1)*N/P), a contiguous byte range of hole, plug and
absmax when K % blocksize == 0, and the outputs are reassembled with one
all-gather where the consumer needs the full row.
"""
from __future__ import annotations

import heapq
from dataclasses import dataclass
from typing import Dict, List, Sequence, Tuple


# Llama-3-8B linear shapes (out_features, in_features) and the embedding
LLAMA3_8B_LAYER = (
    ("q_proj", 4096, 4096), ("k_proj", 1024, 4096), ("v_proj", 1024, 4096), ("o_proj", 4096, 4096),
    ("gate_proj", 14336, 4096), ("up_proj", 14336, 4096), ("down_proj", 4096, 14336),
)
LLAMA3_8B_LAYERS = 32
LLAMA3_8B_EMBED = (128256, 4096)
LLAMA3_70B_LAYER = (
    ("q_proj", 8192, 8192), ("k_proj", 1024, 8192), ("v_proj", 1024, 8192), ("o_proj", 8192, 8192),
    ("gate_proj", 28672, 8192), ("up_proj", 28672, 8192), ("down_proj", 8192, 28672),
)
LLAMA3_70B_LAYERS = 80


@dataclass(frozen=True)
class TensorSpec:
    name: str
    rows: int
    cols: int

    @property
    def numel(self) -> int:
        return self.rows * self.cols


def llama3_8b_tensors() -> List[TensorSpec]:
    """The 225 weights of config 2: 32 layers x 7 linears + the embedding."""
    out = [TensorSpec("model.embed_tokens.weight", *LLAMA3_8B_EMBED)]
    for layer in range(LLAMA3_8B_LAYERS):
        for nm, r, c in LLAMA3_8B_LAYER:
            out.append(TensorSpec(f"model.layers.{layer}.{nm}.weight", r, c))
    return out


def lpt_assign(sizes: Sequence[int], ranks: int) -> List[List[int]]:
    """Indices of `sizes` per rank, largest first onto the least-loaded rank.
    Deterministic: ties go to the lower rank, equal sizes keep input order."""
    if ranks <= 0:
        raise ValueError("ranks must be positive")
    order = sorted(range(len(sizes)), key=lambda i: (-sizes[i], i))
    heap = [(0, r) for r in range(ranks)]
    out: List[List[int]] = [[] for _ in range(ranks)]
    for i in order:
        load, r = heapq.heappop(heap)
        out[r].append(i)
        heapq.heappush(heap, (load + sizes[i], r))
    for lst in out:
        lst.sort()
    return out


def imbalance(sizes: Sequence[int], plan: List[List[int]]) -> float:
    """max rank load / mean rank load."""
    loads = [sum(sizes[i] for i in lst) for lst in plan]
    mean = sum(loads) / len(loads)
    return max(loads) / mean if mean else 1.0


def column_shard(N: int, ranks: int, rank: int, align: int = 16) -> Tuple[int, int]:
    """Row range [n0, n1) of rank `rank` for a column-parallel linear of N outputs,
    boundaries on multiples of `align` rows (the GEMV row tile)."""
    if N % ranks == 0 and (N // ranks) % align == 0:
        step = N // ranks
        return rank * step, (rank + 1) * step
    units = (N + align - 1) // align
    base, extra = divmod(units, ranks)
    u0 = rank * base + min(rank, extra)
    u1 = u0 + base + (1 if rank < extra else 0)
    return min(N, u0 * align), min(N, u1 * align)


def shard_planes(rows: Tuple[int, int], K: int, blocksize: int) -> Dict[str, Tuple[int, int]]:
    """Byte / element ranges of hole, plug (bytes) and absmax (floats) that hold
    packed rows [n0, n1) of a [N, K] weight; needs K * n0 even and on a block edge."""
    n0, n1 = rows
    if (n0 * K) % 2 or (n0 * K) % blocksize:
        raise ValueError("row range does not start on a byte and block boundary")
    return {
        "planes": ((n0 * K) // 2, (n1 * K + 1) // 2),
        "absmax": ((n0 * K) // blocksize, (n1 * K + blocksize - 1) // blocksize),
    }
