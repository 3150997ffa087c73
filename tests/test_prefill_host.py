"""Host logic of the multi-GPU config-4 prefill bench (bench.py --workload prefill): the (batch, head) pairs
are split into contiguous, disjoint, covering shares (no GPU needed)."""
from bench import pair_range


def test_pair_ranges_cover_every_pair_once():
    for n_pairs in (1, 7, 64):
        for world in (1, 2, 3, 4, 8):
            got = [pair_range(n_pairs, r, world) for r in range(world)]
            assert got[0][0] == 0 and got[-1][1] == n_pairs
            for (a0, a1), (b0, b1) in zip(got, got[1:]):
                assert a1 == b0 and a0 <= a1
            sizes = [b - a for a, b in got]
            assert max(sizes) - min(sizes) <= 1
