"""Conjugate-gradient solvers with the reference's API.

Drop-in for ``deepfold.utils.cg`` of the reference (src/deepfold/utils/cg.py):
``conjugate_gradient`` (:28-98) for symmetric positive (semi-)definite systems
and ``steihaug_cg`` (:131-255) for trust-region subproblems, with the frozen
``CGInfo`` / ``SteihaugCGInfo`` reports and the same stopping rules:

* CG stops once ||r|| <= max(atol, rtol * ||r0||) after an update, or when
  p^T A p == 0; ``iters`` counts updates, ``max_iter`` on failure.
* Steihaug stops on convergence, on negative curvature (d^T H d <= tol) or when
  the step leaves the trust region, returning the boundary point.

These solvers take an arbitrary user ``matvec`` and so run a host-driven loop
of tensor operations on whatever device the vectors live on.  The Sinkhorn
backward does not use them: its CG runs entirely on the GPU inside ``dfs_bwd``
(one fused cluster reduction per iteration, no host synchronisation).
"""

from __future__ import annotations

import math
from dataclasses import dataclass
from typing import Callable

import torch

__all__ = ["CGInfo", "conjugate_gradient", "SteihaugCGInfo", "steihaug_cg"]


@dataclass(frozen=True)
class CGInfo:
    """Convergence report of ``conjugate_gradient``."""

    converged: bool
    iters: int
    residual: float
    initial_residual: float


def _norm(v: torch.Tensor) -> float:
    return float(torch.linalg.vector_norm(v).detach().cpu())


def conjugate_gradient(
    matvec: Callable[[torch.Tensor], torch.Tensor],
    b: torch.Tensor,
    *,
    x0: torch.Tensor | None = None,
    max_iter: int = 300,
    rtol: float = 1e-6,
    atol: float = 1e-6,
    preconditioner: Callable[[torch.Tensor], torch.Tensor] | None = None,
    stabilise_every: int = 0,
) -> tuple[torch.Tensor, CGInfo]:
    """Solve A x = b for symmetric positive definite A given ``matvec(v) = A v``.

    ``preconditioner(v)`` applies M^-1; ``stabilise_every = k > 0`` replaces the
    recursive residual by b - A x every k iterations.
    """
    if x0 is None:
        x = torch.zeros_like(b)
        r = b.clone()
    else:
        x = x0.clone()
        r = b - matvec(x)
    apply_m = preconditioner if preconditioner is not None else (lambda v: v)
    z = apply_m(r)
    p = z.clone()
    rz = torch.dot(r, z)
    res0 = _norm(r)
    tol = max(atol, rtol * res0)
    for it in range(int(max_iter)):
        Ap = matvec(p)
        pAp = torch.dot(p, Ap)
        if float(pAp.abs()) == 0.0:
            break
        step = rz / pAp
        x = x + step * p
        r = r - step * Ap
        if stabilise_every and (it + 1) % stabilise_every == 0:
            r = b - matvec(x)
        res = _norm(r)
        if res <= tol:
            return x, CGInfo(converged=True, iters=it + 1, residual=res, initial_residual=res0)
        z = apply_m(r)
        rz_next = torch.dot(r, z)
        p = z + (rz_next / rz) * p
        rz = rz_next
    return x, CGInfo(converged=False, iters=int(max_iter), residual=_norm(r), initial_residual=res0)


@dataclass(frozen=True)
class SteihaugCGInfo:
    """Report of ``steihaug_cg``; ``termination_reason`` is one of
    "converged", "negative_curvature", "boundary", "max_iter"."""

    converged: bool
    iters: int
    residual: float
    termination_reason: str
    hit_boundary: bool
    negative_curvature_detected: bool
    predicted_reduction: float


def _to_boundary(x: torch.Tensor, d: torch.Tensor, delta: float) -> float:
    """Largest-magnitude root tau > 0 of ||x + tau d|| = delta (smallest positive one)."""
    xx = float(torch.dot(x, x))
    xd = float(torch.dot(x, d))
    dd = float(torch.dot(d, d))
    disc = xd * xd - dd * (xx - delta * delta)
    if disc < 0.0:
        return delta / math.sqrt(dd + 1e-10)
    root = math.sqrt(disc)
    t1 = (-xd + root) / (dd + 1e-10)
    t2 = (-xd - root) / (dd + 1e-10)
    if t1 > 0.0 and t2 > 0.0:
        return min(t1, t2)
    hi = max(t1, t2)
    return hi if hi > 0.0 else abs(t1)


def _model_decrease(hvp_fn, grad, step) -> float:
    """-(g^T p + p^T H p / 2) for the quadratic model."""
    return -float(torch.dot(grad, step)) - 0.5 * float(torch.dot(step, hvp_fn(step)))


def steihaug_cg(
    hvp_fn: Callable[[torch.Tensor], torch.Tensor],
    grad: torch.Tensor,
    delta: float,
    *,
    max_iter: int = 100,
    rtol: float = 1e-6,
    atol: float = 1e-6,
    neg_curv_tol: float = 1e-10,
) -> tuple[torch.Tensor, SteihaugCGInfo]:
    """Approximately minimise g^T p + p^T H p / 2 subject to ||p|| <= delta."""
    step = torch.zeros_like(grad)
    r = -grad.clone()
    d = r.clone()
    rnorm = _norm(r)
    tol = max(atol, rtol * rnorm)
    if rnorm < tol:
        return step, SteihaugCGInfo(True, 0, rnorm, "converged", False, False, 0.0)
    neg = False
    for it in range(max_iter):
        Hd = hvp_fn(d)
        dHd = float(torch.dot(d, Hd))
        if dHd <= neg_curv_tol:
            neg = True
            final = step + _to_boundary(step, d, delta) * d
            return final, SteihaugCGInfo(False, it + 1, rnorm, "negative_curvature", True, True,
                                         _model_decrease(hvp_fn, grad, final))
        rr = float(torch.dot(r, r))
        a = rr / dHd
        trial = step + a * d
        if _norm(trial) >= delta:
            final = step + _to_boundary(step, d, delta) * d
            return final, SteihaugCGInfo(False, it + 1, rnorm, "boundary", True, neg,
                                         _model_decrease(hvp_fn, grad, final))
        step = trial
        r = r - a * Hd
        rnorm = _norm(r)
        if rnorm < tol:
            return step, SteihaugCGInfo(True, it + 1, rnorm, "converged", False, neg,
                                        _model_decrease(hvp_fn, grad, step))
        d = r + (float(torch.dot(r, r)) / rr) * d
    return step, SteihaugCGInfo(False, max_iter, rnorm, "max_iter", _norm(step) >= delta * 0.99, neg,
                                _model_decrease(hvp_fn, grad, step))
