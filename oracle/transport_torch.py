"""The reference's balanced Sinkhorn transport, restated in torch.
TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py`` may import this
module; it is the checker for ``balanced_sinkhorn_transport(_dual)``, never the
product.

Reference: src/deepfold/model/kernels/flash_sinkhorn_transport.py of
vv137/deepfold-linear.  It has two paths that differ on padded inputs, and
both are written out here:

* ``transport_device`` -- the device path (Triton kernels, ``:27-243``, driven
  by ``BalancedSinkhornFn.forward`` ``:289-320``), which the trunk block runs:
    C_ij = (1 - w)(1 - q_i.k_j) + w dist_ij / (r + dist_ij),
    dist_ij = sqrt(|x_i - x_j|^2 + 1e-8),  w = sigmoid(alpha_h),
    r = max(|r_h|, 0.1)                                          (:27-54)
    mask bias mb_j = 0 where mask > 0.5 else -1e9; one log marginal for the
    whole batch, the batch mean of -log(max(n_b, 1))             (:293-295)
    K_iter x { log_v = lm - LSE_i(log_u_i - C_ij/eps + mb_i)     (:87-114)
               log_u = lm - LSE_j(-C_ij/eps + log_v_j + mb_j) }  (:57-84)
    T_norm = softmax_j(log_u_i - C_ij/eps + log_v_j + mb_j), every row
    x_centroid = T_norm x, h_centroid = T_norm V                 (:117-243)
  Its gradient here is torch autograd through the K iterations (the
  reference's device backward is the same unrolled gradient written as
  kernels, balanced_sinkhorn_bwd.py:36-404, except that it differentiates
  r_h as if the clamp were the identity).  ``zero_pad_rows`` zeroes the
  padded rows of both outputs, which is what the B200 op returns.

* ``transport_cpu`` -- ``_sinkhorn_cpu`` (``:253-282``), the path the
  reference takes for CPU tensors: dist clamped at 1e-8 instead of the +1e-8
  under the root, the mask folded in as log(mask) on both sides of the log
  kernel, per-sample marginals, T multiplied by the mask on both sides and
  T_norm = T / max(row sum, 1e-8).  With an all-ones mask (or none) both
  paths compute the same transport up to the distance convention (~1e-8).

``tests/test_oracle_transport.py`` pins both against golden vectors that the
reference's own code produced (tests/golden/make_golden.py).
"""

from __future__ import annotations

import torch


def _geometry(x, r, mode):
    diff = x[:, :, None, :] - x[:, None, :, :]
    if mode == "device":
        dist = torch.sqrt((diff * diff).sum(-1) + 1e-8)
    else:
        dist = diff.norm(dim=-1).clamp(min=1e-8)
    return dist[:, None] / (r.view(1, -1, 1, 1) + dist[:, None])


def balanced_cost(Q, K, x, alpha_h, r_h, mode: str = "device"):
    """(B, H, N, N) cosine / geometry cost (flash_sinkhorn_transport.py:27-54)."""
    w = torch.sigmoid(alpha_h.to(Q.dtype)).view(1, -1, 1, 1)
    r = r_h.to(Q.dtype).abs().clamp(min=0.1)
    c_feat = 1.0 - Q @ K.transpose(-1, -2)
    return (1.0 - w) * c_feat + w * _geometry(x.to(Q.dtype), r, mode)


def transport_device(Q, K, x, eps, alpha_h, r_h, K_iter: int = 20, mask=None, V=None,
                     zero_pad_rows: bool = False):
    """Device-path semantics of balanced_sinkhorn_transport(_dual); returns
    x_centroid, or (x_centroid, h_centroid) with V.  Differentiable."""
    B, H, N, _ = Q.shape
    dt = Q.dtype
    logk = -balanced_cost(Q, K, x, alpha_h, r_h, "device") / eps.to(dt).view(1, H, 1, 1)
    if mask is not None:
        valid = mask.to(dt) > 0.5
        mb = torch.where(valid, torch.zeros((), dtype=dt), torch.full((), -1e9, dtype=dt))
        lm = (-torch.log(mask.to(dt).sum(-1).clamp(min=1))).mean()
    else:
        mb = torch.zeros(B, N, dtype=dt)
        lm = -torch.log(torch.tensor(float(N), dtype=dt))
    mb_row = mb[:, None, :, None]   # bias of row i (column update sums over i)
    mb_col = mb[:, None, None, :]   # bias of column j (row update sums over j)
    lu = torch.zeros(B, H, N, dtype=dt)
    lv = torch.zeros(B, H, N, dtype=dt)
    for _ in range(K_iter):
        lv = lm - torch.logsumexp(lu[..., :, None] + logk + mb_row, dim=-2)
        lu = lm - torch.logsumexp(logk + lv[..., None, :] + mb_col, dim=-1)
    tn = torch.softmax(logk + lv[..., None, :] + mb_col, dim=-1)
    xc = tn @ x.to(dt)[:, None]
    hc = tn @ V.to(dt) if V is not None else None
    if zero_pad_rows and mask is not None:
        rows = (mask.to(dt) > 0.5).to(dt)[:, None, :, None]
        xc = xc * rows
        hc = hc * rows if hc is not None else None
    return xc if V is None else (xc, hc)


def transport_cpu(Q, K, x, eps, alpha_h, r_h, K_iter: int = 20, mask=None, V=None):
    """``_sinkhorn_cpu`` (flash_sinkhorn_transport.py:253-282) restated."""
    B, H, N, _ = Q.shape
    dt = Q.dtype
    logk = -balanced_cost(Q, K, x, alpha_h, r_h, "cpu") / eps.to(dt).view(1, H, 1, 1)
    if mask is not None:
        mf = mask.to(dt)
        lmk = torch.log(mf.clamp(min=1e-8))
        logk = logk + lmk[:, None, :, None] + lmk[:, None, None, :]
        lm = -torch.log(mf.sum(-1, keepdim=True).clamp(min=1))[:, None, :, None]   # (B,1,1,1)
    else:
        lm = -torch.log(torch.tensor(float(N), dtype=dt))
    lu = torch.zeros(B, H, N, 1, dtype=dt)
    lv = torch.zeros(B, H, 1, N, dtype=dt)
    for _ in range(K_iter):
        lv = lm - torch.logsumexp(logk + lu, dim=-2, keepdim=True)
        lu = lm - torch.logsumexp(logk + lv, dim=-1, keepdim=True)
    T = (lu + logk + lv).exp()
    if mask is not None:
        T = T * mask.to(dt).view(B, 1, N, 1) * mask.to(dt).view(B, 1, 1, N)
    tn = T / T.sum(-1, keepdim=True).clamp(min=1e-8)
    xc = torch.einsum("bhij,bjc->bhic", tn, x.to(dt))
    if V is None:
        return xc
    return xc, torch.einsum("bhij,bhjd->bhid", tn, V.to(dt))


def transport_grads(fn, Q, K, x, eps, alpha_h, r_h, V=None, gxc=None, ghc=None, **kw):
    """Outputs and the gradients of sum(gxc * x_centroid) + sum(ghc * h_centroid)
    with respect to Q, K, x, V, alpha_h, r_h (torch autograd through ``fn``)."""
    leaves = [t.detach().clone().requires_grad_(True) for t in (Q, K, x, alpha_h, r_h)]
    vl = V.detach().clone().requires_grad_(True) if V is not None else None
    out = fn(leaves[0], leaves[1], leaves[2], eps, leaves[3], leaves[4], V=vl, **kw)
    xc, hc = (out, None) if V is None else out
    loss = (xc * gxc).sum() if gxc is not None else xc.sum() * 0
    if hc is not None and ghc is not None:
        loss = loss + (hc * ghc).sum()
    wrt = leaves + ([vl] if vl is not None else [])
    g = torch.autograd.grad(loss, wrt, allow_unused=True)
    names = ["dQ", "dK", "dx", "dalpha", "dr"] + (["dV"] if vl is not None else [])
    res = {n: (t if t is not None else torch.zeros_like(w)) for n, t, w in zip(names, g, wrt)}
    res["xc"] = xc.detach()
    if hc is not None:
        res["hc"] = hc.detach()
    return res
