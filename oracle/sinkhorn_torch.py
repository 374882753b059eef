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
* ``compute_bins``              -- position_encoding.py:7-52 (the pair bins the
         position term gathers)

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


def compute_bins(chain_id, global_idx, bond_matrix):
    """position_encoding.py:7-52: the 68-bin position / bond code of every pair,
    (N, N) or (B, N, N) int32."""
    unb = chain_id.dim() == 1
    if unb:
        chain_id, global_idx, bond_matrix = chain_id[None], global_idx[None], bond_matrix[None]
    same = chain_id[:, :, None] == chain_id[:, None, :]
    bond = bond_matrix.bool()
    sep = (global_idx[:, :, None] - global_idx[:, None, :]).clamp(-32, 32) + 32
    bins = torch.where(bond, torch.where(same, 66, 67), torch.where(same, sep, 65)).to(torch.int32)
    return bins[0] if unb else bins


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
            ch = max(float((log_u - u_prev).detach().abs().max()), float((log_v - v_prev).detach().abs().max()))
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


# --------------------------------------------------------------------------
# one problem, float64, implicit-function-theorem adjoint (no autograd state)
# --------------------------------------------------------------------------

def problem_fwd_bwd_ift(q, k, v, dO, eps: float, a, b, K_iter: int, lam: float, mask=None, cg_tol=1e-12,
                        cg_max_iter=2000):
    """Forward and gradient of sum(O * dO) for one (N, d) problem, in the dtype of
    its inputs (float64 for checking), without autograd: the reference's loop
    (sinkhorn.py:82-96) and transport (sinkhorn.py:152-195), then the
    transport adjoint and the implicit-function-theorem adjoint of the fixed
    point -- the same formulation as oracle/sinkhorn_oracle.py's
    transport_backward / ift_backward, for problems (N = 8192) whose unrolled
    autograd state would not fit in host memory.  At a converged forward it
    equals the reference's unrolled gradient.

    Returns dict(O, log_u, log_v, dQ, dK, dV, marg_row, marg_col)."""
    N, d = q.shape
    kap = 1.0 if math.isinf(lam) else lam / (lam + eps)
    valid = torch.ones(N, dtype=torch.bool) if mask is None else mask > 0.5
    mb = torch.zeros(N, dtype=q.dtype) if mask is None else (1.0 - mask.to(q.dtype)) * MASK_BIAS
    S = (q @ k.T) / (math.sqrt(d) * eps)          # S = -C / eps
    f = torch.zeros(N, dtype=q.dtype)
    g = torch.zeros(N, dtype=q.dtype)
    for _ in range(K_iter):
        f = kap * (a - torch.logsumexp(S + (g + mb)[None, :], dim=1))
        g = kap * (b - torch.logsumexp(S + (f + mb)[:, None], dim=0))
    # transport (running max over masked columns, 1e-6 in the normaliser)
    score = f[:, None] + S + (g + mb)[None, :]
    m, am = score.max(dim=1, keepdim=True)
    T = torch.exp(score - m)
    del score
    Ts = T.sum(1)
    den = Ts + NORM_EPS
    Tn = T / den[:, None]
    Tn = Tn * valid[:, None]
    O = Tn @ v
    # transport adjoint: dS_direct, df = row sums, dg = column sums, dV
    dOm = dO * valid[:, None]
    Tbar_n = (dOm @ v.T) * valid[:, None]
    dV = Tn.T @ dOm
    del Tn
    Tbar = Tbar_n / den[:, None] - ((Tbar_n * T).sum(1) / den ** 2)[:, None]
    del Tbar_n
    sbar = Tbar * T
    # the row maximum's own term (nonzero only through the 1e-6 of the normaliser)
    sbar.scatter_add_(1, am, -(Tbar * T).sum(1, keepdim=True))
    del Tbar, T
    df, dg = sbar.sum(1), sbar.sum(0)
    # IFT system [[diag(r)/kappa, P], [P^T, diag(c)/kappa]] w = [df; dg]
    P = torch.exp(f[:, None] + S + g[None, :]) * valid[:, None] * valid[None, :]
    r, c = P.sum(1), P.sum(0)
    dr = torch.where(valid, r / kap, torch.ones_like(r))
    dc = torch.where(valid, c / kap, torch.ones_like(c))
    rhs = torch.cat([torch.where(valid, df, 0 * df), torch.where(valid, dg, 0 * dg)])
    nv = int(valid.sum())
    if kap >= 1.0 and nv > 0:
        s = (rhs[:N][valid].sum() - rhs[N:][valid].sum()) / (2 * nv)
        rhs[:N] = torch.where(valid, rhs[:N] - s, rhs[:N])
        rhs[N:] = torch.where(valid, rhs[N:] + s, rhs[N:])

    def mv(w):
        return torch.cat([dr * w[:N] + P @ w[N:], P.T @ w[:N] + dc * w[N:]])

    dinv = 1.0 / torch.cat([dr, dc])
    w = torch.zeros(2 * N, dtype=q.dtype)
    res = rhs.clone()
    z = dinv * res
    p = z.clone()
    rz = res @ z
    nrm0 = float(torch.linalg.norm(res))
    for _ in range(cg_max_iter):
        if nrm0 == 0.0:
            break
        Ap = mv(p)
        dd = float(p @ Ap)
        if dd == 0.0:
            break
        al = rz / dd
        w = w + al * p
        res = res - al * Ap
        if float(torch.linalg.norm(res)) <= cg_tol * nrm0:
            break
        z = dinv * res
        rz_new = res @ z
        p = z + (rz_new / rz) * p
        rz = rz_new
    w1, w2 = w[:N] * valid, w[N:] * valid
    if kap >= 1.0 and nv > 0:
        t = -(r * w1).sum() / r.sum()
        w1 = (w1 + t) * valid
        w2 = (w2 - t) * valid
    dS = sbar - P * (w1[:, None] + w2[None, :])
    del sbar
    marg_r = float(((r - a.exp()).abs() * valid).max())
    marg_c = float(((c - b.exp()).abs() * valid).max())
    del P
    dC_scale = 1.0 / (math.sqrt(d) * eps)          # dS/dQ = K / (sqrt(d) eps)
    dQ = (dS @ k) * dC_scale
    dK = (dS.T @ q) * dC_scale
    fo = f * valid
    go = g * valid
    return dict(O=O, log_u=fo, log_v=go, dQ=dQ, dK=dK, dV=dV, marg_row=marg_r, marg_col=marg_c)
