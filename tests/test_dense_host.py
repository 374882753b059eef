"""Host logic of the differentiable dense solve (deepfold/model/sinkhorn.py):
where it returns to the host to apply the reference's batch-wide early stop.
The reference tests max(|du|, |dv|) < threshold after every check_every-th
iteration (src/deepfold/model/sinkhorn.py:98-103); the forward must stop at the
same iteration so that the adjoint covers exactly the iterations the reference
runs.  No GPU needed."""

import pytest

from deepfold.model.sinkhorn import _chunk_ends, _is_check


def reference_checks(K, check_every):
    """Iteration counts (1-based) after which the reference's loop tests."""
    return [i + 1 for i in range(K) if (i + 1) % check_every == 0]


@pytest.mark.parametrize("K,every", [(7, 2), (10, 5), (9, 3), (1, 2), (0, 2), (40, 1)])
def test_chunks_end_at_every_reference_check_and_at_K(K, every):
    ends = _chunk_ends(K, 1e-3, every)
    assert ends == sorted(set(ends)) and (not ends or ends[-1] == K)
    checks = [e for e in ends if _is_check(e, 1e-3, every)]
    assert checks == reference_checks(K, every)
    # nothing but the checks and K
    assert set(ends) - set(checks) <= {K}


def test_no_threshold_is_one_chunk_without_checks():
    assert _chunk_ends(20, None, 2) == [20]
    assert not _is_check(20, None, 2)


def test_stop_iteration_matches_a_simulated_reference_loop():
    """A change sequence that falls below the threshold at iteration 6: the
    reference (check_every = 3) stops after 6; so does the chunked forward."""
    changes = {i: 10.0 ** (-i) for i in range(1, 13)}
    thr, every, K = 2e-6, 3, 12
    ref_stop = next(i + 1 for i in range(K) if (i + 1) % every == 0 and changes[i + 1] < thr)
    stop = None
    for end in _chunk_ends(K, thr, every):
        stop = end
        if _is_check(end, thr, every) and changes[end] < thr:
            break
    assert stop == ref_stop == 6
