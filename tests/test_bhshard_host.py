"""(batch, head) partition of the padded var-len configuration (B=8, H=16, N=1024) on CPU: every problem once,
contiguous head ranges, and a cost imbalance of at most one problem."""

import random

import pytest

from deepfold.model.kernels.sinkhorn_bhshard import partition_problems, rank_blocks


@pytest.mark.parametrize("world", [1, 2, 3, 4, 8])
def test_partition_covers_balances_and_keeps_views_contiguous(world):
    rng = random.Random(world)
    for _ in range(20):
        B, H = rng.randint(1, 9), rng.choice([1, 4, 16])
        lengths = [rng.randint(64, 1024) for _ in range(B)]
        parts = partition_problems(lengths, H, world)
        assert len(parts) == world
        seen = set()
        loads = []
        for chunks in parts:
            load = 0
            for b, h0, h1 in chunks:
                assert 0 <= b < B and 0 <= h0 < h1 <= H
                for h in range(h0, h1):
                    assert (b, h) not in seen
                    seen.add((b, h))
                load += (h1 - h0) * lengths[b] ** 2
            loads.append(load)
        assert seen == {(b, h) for b in range(B) for h in range(H)}
        total = sum(loads)
        biggest = max(lengths) ** 2
        assert max(loads) <= total / world + biggest + 1e-9


@pytest.mark.parametrize("world", [1, 2, 3, 8])
def test_rank_blocks_are_rectangles_of_the_sorted_batch(world):
    rng = random.Random(100 + world)
    for _ in range(20):
        B, H = rng.randint(1, 9), rng.choice([1, 4, 16])
        lengths = [rng.randint(64, 1024) for _ in range(B)]
        covered = set()
        for r in range(world):
            order, blocks = rank_blocks(lengths, H, world, r)
            assert sorted(order) == list(range(B))
            assert all(lengths[order[i]] >= lengths[order[i + 1]] for i in range(B - 1))
            assert len(blocks) <= 3
            for s0, s1, h0, h1 in blocks:
                assert s0 < s1 and h0 < h1 and (s1 - s0 == 1 or (h0, h1) == (0, H))
                for sp in range(s0, s1):
                    for h in range(h0, h1):
                        assert (order[sp], h) not in covered
                        covered.add((order[sp], h))
        assert covered == {(b, h) for b in range(B) for h in range(H)}
