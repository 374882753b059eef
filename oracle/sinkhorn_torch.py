"""The reference's PyTorch CPU path for the flash-Sinkhorn operator, restated.
TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` (its
``cpu_baseline`` leg and the ``--impl reference`` arm) may import this module.
It is the checker and the timed CPU baseline, never the product: the shipped
path is the CUDA library behind ``include/dfsink.h``.

The reference (vv137/deepfold-linear) differentiates its dense path with torch
autograd; that dense path is what its own gradient tests compare against
(tests/test_triton_fallback_consistency.py:316-355) and what a CPU user of the
reference runs.  The reference source cannot be shipped with this repository,
so the same torch computation is written out here:

* cost   C = -Q K^T / sqrt(d) + pos_weight[h, bins] + w_h * dist/(r_0 + dist),
         dist = sqrt(|x_i - x_j|^2 + 1e-8)   -- sinkhorn_kernel.py:59-129
* ``sinkhorn_solve``            -- sinkhorn.py:17-112 (row then column update,
         kappa = lam/(lam+eps), -1e9 mask biases, optional L-inf early stop,
         padded duals zeroed)
* ``compute_transport_output``  -- sinkhorn.py:115-198 (running-max plan,
         T / (sum T + 1e-6), padded rows zeroed, sigmoid(G) gate, centroid)
* gradients: torch autograd through all of it, exactly as the reference does.

One deliberate extension: ``lam = inf`` gives kappa = 1 (the reference's
lam/(lam+eps) is NaN there); callers that want the reference's own arithmetic
pass lam = 1e6.  ``tests/test_oracle_torch.py`` pins this file against the
golden vectors in ``tests/golden`` (produced by the reference's own code).
"""

from __future__ import annotations

import math

import torch

MASK_BIAS = -1e9
NORM_EPS = 1e-6


def kappa_of(lam: float, eps: torch.Tensor) -> torch.Tensor:
    if math.isinf(lam):
        return torch.ones_like(eps)
    return lam / (lam + eps)


def cost(Q, K, x=None, pos_weight=None, bins=None, w_dist=None, r_0: float = 10.0):
    """(B, H, N, N) cost of sinkhorn_kernel.py:59-129 (terms absent when None)."""
    d = Q.shape[-1]
    C = -(Q @ K.transpose(-1, -2)) / math.sqrt(d)
    if x is not None and w_dist is not None:
        diff = x[:, :, None, :] - x[:, None, :, :]
        dist = torch.sqrt((diff * diff).sum(-1) + 1e-8)
        C = C + w_dist[None, :, None, None] * (dist / (r_0 + dist))[:, None]
    if pos_weight is not None and bins is not None:
        C = C + pos_weight[:, bins.long()].permute(1, 0, 2, 3)
    return C


def sinkhorn_solve(C, log_mu, log_nu, eps, lam=1.0, K=7, log_u_init=None, log_v_init=None, threshold=None,
                   check_every=2, mask=None):
    """sinkhorn.py:17-112 on (B, H, N, N) costs."""
    kappa = kappa_of(lam, eps)
    log_u = log_u_init if log_u_init is not None else torch.zeros_like(log_mu)
    log_v = log_v_init if log_v_init is not None else torch.zeros_like(log_nu)
    log_K = -C / eps[None, :, None, None]
    if mask is not None:
        mf = mask.to(C.dtype)
        col_bias = (1 - mf)[:, None, None, :] * MASK_BIAS
        row_bias = (1 - mf)[:, None, :, None] * MASK_BIAS
    else:
        col_bias = row_bias = 0
    for i in range(K):
        u_prev, v_prev = log_u, log_v
        log_u = kappa[None, :, None] * (log_mu - torch.logsumexp(log_K + log_v[:, :, None, :] + col_bias, dim=-1))
        log_v = kappa[None, :, None] * (log_nu - torch.logsumexp(log_K + log_u[:, :, :, None] + row_bias, dim=-2))
        if threshold is not None and (i + 1) % check_every == 0:
            ch = max(float((log_u - u_prev).abs().max()), float((log_v - v_prev).abs().max()))
            if ch < threshold:
                break
    if mask is not None:
        log_u = log_u * mask[:, None, :]
        log_v = log_v * mask[:, None, :]
    return log_u, log_v


def compute_transport_output(V, G, log_u, log_v, C, eps, x_res=None, mask=None):
    """sinkhorn.py:115-198 on batched inputs: (o (B, N, H*d), T_norm, x_centroid, O_avg)."""
    log_score = log_u[:, :, :, None] + (-C / eps[None, :, None, None]) + log_v[:, :, None, :]
    if mask is not None:
        mf = mask.to(C.dtype)
        log_score = log_score + (1 - mf)[:, None, None, :] * MASK_BIAS
    T = torch.exp(log_score - log_score.max(dim=-1, keepdim=True).values)
    T_norm = T / (T.sum(dim=-1, keepdim=True) + NORM_EPS)
    if mask is not None:
        T_norm = T_norm * mf[:, None, :, None]
    O_avg = T_norm @ V
    o = O_avg if G is None else torch.sigmoid(G) * O_avg
    B, H, N, d = o.shape
    o = o.permute(0, 2, 1, 3).reshape(B, N, H * d)
    if mask is not None:
        o = o * mf[:, :, None]
    xc = None if x_res is None else torch.einsum("bhnm,bmc->bhnc", T_norm, x_res)
    return o, T_norm, xc, O_avg


def attn(Q, K, V, eps, log_mu, log_nu, K_iter, lam, G=None, x_res=None, pos_weight=None, bins=None, w_dist=None,
         r_0=10.0, mask=None):
    """Dense forward of flash_sinkhorn_attn as the reference's CPU user runs it:
    cost, sinkhorn_solve, compute_transport_output.  Returns (o_flat, O_avg,
    x_centroid, log_u, log_v)."""
    C = cost(Q, K, x_res, pos_weight, bins, w_dist, r_0)
    lu, lv = sinkhorn_solve(C, log_mu, log_nu, eps, lam=lam, K=K_iter, mask=mask)
    o, _, xc, O_avg = compute_transport_output(V, G, lu, lv, C, eps, x_res=x_res, mask=mask)
    return o, O_avg, xc, lu, lv


def attn_fwd_bwd(Q, K, V, eps, log_mu, log_nu, K_iter, lam, dO, dtype=torch.float32, **kw):
    """Forward plus autograd backward of sum(O_avg * dO) on copies of Q, K, V in
    ``dtype``; returns (O_avg, log_u, log_v, dQ, dK, dV)."""
    leaves = [t.detach().to(dtype).requires_grad_(True) for t in (Q, K, V)]
    cast = lambda t: None if t is None else t.to(dtype)  # noqa: E731
    _, O_avg, _, lu, lv = attn(*leaves, cast(eps), cast(log_mu), cast(log_nu), K_iter, lam,
                               **{k: (cast(v) if isinstance(v, torch.Tensor) and v.is_floating_point() else v)
                                  for k, v in kw.items()})
    dQ, dK, dV = torch.autograd.grad(O_avg, leaves, grad_outputs=dO.to(dtype))
    return O_avg.detach(), lu.detach(), lv.detach(), dQ, dK, dV


def marginal_residuals(Q, K, eps, log_u, log_v, log_mu, log_nu, mask=None):
    """max |P 1 - mu| and max |P^T 1 - nu| of P = exp(f + S + g) over valid entries
    (float64), per (B, H) batch."""
    d = Q.shape[-1]
    S = (Q.double() @ K.double().transpose(-1, -2)) / math.sqrt(d) / eps.double()[None, :, None, None]
    P = torch.exp(log_u.double()[..., :, None] + S + log_v.double()[..., None, :])
    if mask is not None:
        m = mask.double()
        P = P * m[:, None, :, None] * m[:, None, None, :]
        valid = m[:, None, :] > 0
    else:
        valid = torch.ones_like(log_mu, dtype=torch.bool)
    r = (P.sum(-1) - log_mu.double().exp()).abs().masked_fill(~valid, 0)
    c = (P.sum(-2) - log_nu.double().exp()).abs().masked_fill(~valid, 0)
    return float(r.max()), float(c.max())
