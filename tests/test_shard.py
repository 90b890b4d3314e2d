"""Host-side placement logic (glint_b200/shard.py), property-tested on the CPU.

- column_shard: the ranks' row ranges tile [0, N) in rank order, on multiples of
  the 16-row tile, with at most one tile of difference between ranks (ranks
  beyond the number of tiles get [N, N));
- shard_planes: for K % blocksize == 0 the ranks' plane byte ranges and absmax
  ranges tile the whole tensor's, so a rank's shard is one contiguous slice;
- lpt_assign: every tensor on exactly one rank, deterministic, and the largest
  rank load within one tensor of the mean (the LPT bound used for encode's weak
  scaling)."""
from hypothesis import given, settings
from hypothesis import strategies as st

from glint_b200 import shard


@settings(max_examples=300, deadline=None)
@given(N=st.integers(1, 200000), ranks=st.integers(1, 8))
def test_column_shard_tiles_rows(N, ranks):
    ranges = [shard.column_shard(N, ranks, r) for r in range(ranks)]
    assert ranges[0][0] == 0 and ranges[-1][1] == N
    for (a0, a1), (b0, b1) in zip(ranges, ranges[1:]):
        assert a1 == b0
    for n0, n1 in ranges:
        # a rank left without a tile gets the empty range [N, N)
        assert n0 <= n1 and (n0 % 16 == 0 or n0 == N) and (n1 % 16 == 0 or n1 == N)
    tiles = [(n1 - n0 + 15) // 16 for n0, n1 in ranges]
    assert max(tiles) - min(tiles) <= 1


@settings(max_examples=300, deadline=None)
@given(N=st.integers(1, 50000), kb=st.integers(1, 64), bs=st.sampled_from([16, 32, 64, 128]),
       ranks=st.integers(1, 8))
def test_shard_planes_tile_the_tensor(N, kb, bs, ranks):
    K = kb * bs
    parts = [shard.shard_planes(shard.column_shard(N, ranks, r), K, bs) for r in range(ranks)]
    planes = [p["planes"] for p in parts]
    am = [p["absmax"] for p in parts]
    assert planes[0][0] == 0 and planes[-1][1] == (N * K + 1) // 2
    assert am[0][0] == 0 and am[-1][1] == (N * K + bs - 1) // bs
    for (a0, a1), (b0, b1) in zip(planes, planes[1:]):
        assert a1 == b0
    for (a0, a1), (b0, b1) in zip(am, am[1:]):
        assert a1 == b0


@settings(max_examples=200, deadline=None)
@given(sizes=st.lists(st.integers(0, 10 ** 9), min_size=0, max_size=300), ranks=st.integers(1, 8))
def test_lpt_assign_places_every_tensor_once(sizes, ranks):
    plan = shard.lpt_assign(sizes, ranks)
    assert plan == shard.lpt_assign(sizes, ranks)
    flat = sorted(i for lst in plan for i in lst)
    assert flat == list(range(len(sizes)))
    loads = [sum(sizes[i] for i in lst) for lst in plan]
    if sizes:
        assert max(loads) <= sum(sizes) / ranks + max(sizes)


def test_lpt_balances_the_benchmark_model():
    """The 225 tensors of the Llama-3-8B-shaped job over 2, 4 and 8 ranks (one model
    copy per rank): within 1 % of perfect balance."""
    specs = shard.llama3_8b_tensors()
    for world in (2, 4, 8):
        job = [s.numel for _ in range(world) for s in specs]
        assert shard.imbalance(job, shard.lpt_assign(job, world)) < 1.01
