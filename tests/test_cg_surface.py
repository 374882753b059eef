"""``deepfold.utils.cg`` against the reference's solver tests, restated.

The reference pins ``conjugate_gradient`` and ``steihaug_cg`` with
tests/test_cg.py:9-100 (identity system, SPD system against a direct solve,
warm start, Jacobi preconditioner; Steihaug: zero gradient, interior SPD
solution, negative curvature, trust-region boundary).  The same checks run here
on the CPU (the solvers are host-side torch code that takes any matvec).
``test_warm_start`` of the reference fails on the reference itself (31 > 30
iterations for that seed); the restatement below checks the property the test
aims at -- a warm start near the solution needs no more iterations than a cold
one -- on a well-conditioned system where it holds for both implementations.
"""

import pytest
import torch

from deepfold.utils.cg import CGInfo, SteihaugCGInfo, conjugate_gradient, steihaug_cg


def _spd(n, shift, seed):
    g = torch.Generator().manual_seed(seed)
    A = torch.randn(n, n, generator=g)
    return A.T @ A + shift * torch.eye(n), torch.randn(n, generator=g)


def test_identity_system():
    b = torch.tensor([1.0, 2.0, 3.0])
    x, info = conjugate_gradient(lambda v: v, b, max_iter=10)
    assert isinstance(info, CGInfo) and info.converged and info.iters <= 1
    assert torch.allclose(x, b, atol=1e-5)


def test_spd_system_matches_direct_solve():
    A, b = _spd(20, 0.1, 42)
    x, info = conjugate_gradient(lambda v: A @ v, b, max_iter=50)
    assert info.converged
    assert torch.allclose(x, torch.linalg.solve(A, b), atol=1e-4)


def test_warm_start_needs_no_more_iterations():
    A, b = _spd(20, 5.0, 7)
    x_true = torch.linalg.solve(A, b)
    _, cold = conjugate_gradient(lambda v: A @ v, b, max_iter=100)
    x0 = x_true + 1e-3 * torch.randn(20, generator=torch.Generator().manual_seed(8))
    _, warm = conjugate_gradient(lambda v: A @ v, b, x0=x0, max_iter=100)
    assert warm.converged and warm.iters <= cold.iters


def test_jacobi_preconditioner_needs_no_more_iterations():
    A = torch.diag(torch.linspace(0.1, 10.0, 20))
    b = torch.randn(20, generator=torch.Generator().manual_seed(42))
    _, plain = conjugate_gradient(lambda v: A @ v, b, max_iter=50)
    _, pre = conjugate_gradient(lambda v: A @ v, b, max_iter=50, preconditioner=lambda v: v / torch.diag(A))
    assert pre.iters <= plain.iters


def test_steihaug_zero_gradient():
    p, info = steihaug_cg(lambda v: v, torch.zeros(5), delta=1.0)
    assert isinstance(info, SteihaugCGInfo) and info.converged and info.iters == 0
    assert torch.count_nonzero(p) == 0


def test_steihaug_interior_solution():
    H, g = _spd(10, 0.5, 42)
    p, info = steihaug_cg(lambda v: H @ v, g, delta=100.0, max_iter=50)
    assert info.converged and not info.hit_boundary
    assert torch.allclose(p, -torch.linalg.solve(H, g), atol=1e-3)


def test_steihaug_negative_curvature():
    H = torch.diag(torch.tensor([1.0, -1.0, 1.0]))
    p, info = steihaug_cg(lambda v: H @ v, torch.tensor([0.0, 1.0, 0.0]), delta=1.0, max_iter=50)
    assert info.hit_boundary or info.negative_curvature_detected


def test_steihaug_trust_region_boundary():
    p, info = steihaug_cg(lambda v: v, torch.tensor([10.0, 0.0]), delta=1.0, max_iter=50)
    assert info.hit_boundary
    assert abs(float(torch.linalg.norm(p)) - 1.0) < 0.02


@pytest.mark.parametrize("dtype", [torch.float32, torch.float64])
def test_cg_keeps_the_input_dtype(dtype):
    A, b = _spd(8, 1.0, 3)
    x, info = conjugate_gradient(lambda v: A.to(dtype) @ v, b.to(dtype), max_iter=40)
    assert x.dtype == dtype and info.converged
