"""(batch, head) partition of BASELINE config 3 on CPU: every problem once,
contiguous head ranges, and a cost imbalance of at most one problem."""

import random

import pytest

from deepfold.model.kernels.sinkhorn_bhshard import partition_problems


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
