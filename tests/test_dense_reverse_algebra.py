"""The algebra of the dense solve's reverse pass (csrc/dfs_dense_grad.cu),
restated in float64 torch and checked against autograd through the reference's
loop (oracle/sinkhorn_torch.py, a restatement of src/deepfold/model/sinkhorn.py:
17-112).  No GPU: this pins the formulas the kernels implement -- softmax
weights recovered from stored potentials, the adjoint recurrences, and the
cost gradient as the shifted rank-2K product of row and column factors -- so a
kernel bug and a derivation error cannot hide behind one another.
"""

import math

import pytest
import torch

from oracle import sinkhorn_torch as ort

MASK_BIAS = -1e9


def forward_history(C, mu, nu, eps, lam, K, lvi, mask):
    """The iterates u_i, v_i (i = 0..K) of the reference's loop, unmasked."""
    kap = (torch.ones_like(eps) if math.isinf(lam) else lam / (lam + eps))[None, :, None]
    L = -C / eps[None, :, None, None]
    cb = rb = 0.0
    if mask is not None:
        cb = (1 - mask)[:, None, None, :] * MASK_BIAS
        rb = (1 - mask)[:, None, :, None] * MASK_BIAS
    us, vs = [torch.zeros_like(mu)], [lvi.clone()]
    for _ in range(K):
        u = kap * (mu - torch.logsumexp(L + vs[-1][:, :, None, :] + cb, -1))
        v = kap * (nu - torch.logsumexp(L + u[:, :, :, None] + rb, -2))
        us.append(u)
        vs.append(v)
    return us, vs, kap, L, cb, rb


def reverse(C, mu, nu, eps, lam, K, lvi, mask, g_lu, g_lv):
    """The reverse as the kernels run it: rev_row / rev_col (or rev_fused)
    recurrences, then the factored cost-gradient pass."""
    us, vs, kap, L, cb, rb = forward_history(C, mu, nu, eps, lam, K, lvi, mask)
    mk = 1.0 if mask is None else mask[:, None, :]
    gv = {K: g_lv * mk}       # gv_K: the masked upstream adjoint of v_K
    gu = {}
    dmu = torch.zeros_like(mu)
    dnu = kap * gv[K]
    for i in range(K, 0, -1):
        # Pc_rj = exp(Y_rj - b_j + v_i,j / kappa): the column softmax recovered from v_i
        Pc = torch.exp(L + us[i][:, :, :, None] + rb + (vs[i] / kap - nu)[:, :, None, :])
        gu[i] = (g_lu * mk if i == K else 0.0) - kap * (gv[i][:, :, None, :] * Pc).sum(-1)
        dmu = dmu + kap * gu[i]
        # Pr_rj = exp(X_rj - a_r + u_i,r / kappa): the row softmax recovered from u_i
        Pr = torch.exp(L + vs[i - 1][:, :, None, :] + cb + (us[i] / kap - mu)[:, :, :, None])
        gv[i - 1] = -kap * (gu[i][:, :, :, None] * Pr).sum(-2)
        if i > 1:
            dnu = dnu + kap * gv[i - 1]
    # the cost gradient as a shifted rank-2K product (dense_dc_fact_kernel):
    # dC = kappa/eps [exp2(c sc + s + t) sum_i A_i B_i + exp2(c sc + s' + t') sum_i A'_i B'_i]
    l2e = 1.0 / math.log(2.0)
    sc = (-l2e / eps)[None, :, None, None]
    U = torch.stack([us[i] * l2e for i in range(1, K + 1)])                    # rows, column-softmax term
    Ur = torch.stack([(us[i] / kap - mu) * l2e for i in range(1, K + 1)])       # rows, row-softmax term
    Vc = torch.stack([(vs[i] / kap - nu) * l2e for i in range(1, K + 1)])       # columns, column-softmax term
    Vr = torch.stack([vs[i - 1] * l2e for i in range(1, K + 1)])                # columns, row-softmax term
    s, s1, t, t1 = U.max(0).values, Ur.max(0).values, Vc.max(0).values, Vr.max(0).values
    w = torch.stack([gv[i] for i in range(1, K + 1)])
    w1 = torch.stack([gu[i] for i in range(1, K + 1)])
    A = torch.exp2(U - s)
    A1 = w1 * torch.exp2(Ur - s1)
    Bf = w * torch.exp2(Vc - t)
    B1 = torch.exp2(Vr - t1)
    S1 = torch.einsum("kbhr,kbhj->bhrj", A, Bf)
    S2 = torch.einsum("kbhr,kbhj->bhrj", A1, B1)
    c2 = C * sc
    dC = (kap / eps[None, :, None])[..., None] * (
        torch.exp2(c2 + s[..., :, None] + t[..., None, :]) * S1
        + torch.exp2(c2 + s1[..., :, None] + t1[..., None, :]) * S2)
    if mask is not None:  # padded rows and columns exactly 0, as autograd gives them
        dC = dC * mask[:, None, :, None] * mask[:, None, None, :]
    return dict(dC=dC, dmu=dmu, dnu=dnu, dlvi=gv[0])


@pytest.mark.parametrize("lam", [1.0, math.inf])
@pytest.mark.parametrize("masked", [False, True])
def test_reverse_algebra_matches_autograd(lam, masked):
    g = torch.Generator().manual_seed(3)
    B, H, N, K = 2, 2, 23, 6
    C = torch.rand(B, H, N, N, generator=g, dtype=torch.float64)
    C = C + C.transpose(-1, -2)
    mask = None
    z = torch.randn(2, B, H, N, generator=g, dtype=torch.float64)
    if masked:
        mask = torch.ones(B, N, dtype=torch.float64)
        mask[1, 15:] = 0
        z = torch.where(mask[None, :, None, :] > 0, z, torch.full_like(z, -1e30))
    lm = torch.log_softmax(z, -1)
    if masked:  # the reference's padding of the marginals (tests/test_sinkhorn_batch.py:59-62)
        lm = torch.where(mask[None, :, None, :] > 0, lm, torch.full_like(lm, -1e9))
    mu, nu = lm[0], lm[1]
    eps = torch.tensor([0.5, 2.0], dtype=torch.float64)
    lvi = 0.3 * torch.randn(B, H, N, generator=g, dtype=torch.float64)
    g_lu, g_lv = (torch.randn(B, H, N, generator=g, dtype=torch.float64) for _ in range(2))

    leaves = [t.clone().requires_grad_(True) for t in (C, mu, nu, lvi)]
    lu, lv = ort.sinkhorn_solve(leaves[0], leaves[1], leaves[2], eps, lam=lam, K=K, log_v_init=leaves[3],
                                mask=mask)
    ((lu * g_lu).sum() + (lv * g_lv).sum()).backward()
    ref = dict(dC=leaves[0].grad, dmu=leaves[1].grad, dnu=leaves[2].grad, dlvi=leaves[3].grad)

    got = reverse(C, mu, nu, eps, lam, K, lvi, mask, g_lu, g_lv)
    for k in ref:
        scale = float(ref[k].abs().max())
        err = float((got[k] - ref[k]).abs().max())
        assert err <= 1e-9 * max(scale, 1.0), (k, err, scale)
    if masked:
        assert float(got["dC"][1, :, 15:, :].abs().max()) == 0.0
        assert float(ref["dC"][1, :, 15:, :].abs().max()) == 0.0


@pytest.mark.parametrize("masked", [False, True])
def test_transport_backward_algebra_matches_autograd(masked):
    """compute_transport_output's backward as dfs_dense_transport_bwd forms it:
    dL/dT_norm from plain products, dscore = Tn (dTn - <dTn, Tn>_row), dC =
    -dscore / eps, dlog_v = column sums, dlog_u = 0 -- against float64 autograd
    through the reference's formulas (sinkhorn.py:152-194), whose rowmax path
    contributes a 1e-6-relative term that the kernels drop."""
    g = torch.Generator().manual_seed(8)
    B, H, N, d = 2, 2, 19, 5
    C = torch.rand(B, H, N, N, generator=g, dtype=torch.float64) * 2
    lu = torch.randn(B, H, N, generator=g, dtype=torch.float64)
    lv = torch.randn(B, H, N, generator=g, dtype=torch.float64)
    V = torch.randn(B, H, N, d, generator=g, dtype=torch.float64)
    x = torch.randn(B, N, 3, generator=g, dtype=torch.float64)
    eps = torch.tensor([0.5, 2.0], dtype=torch.float64)
    mask = None
    if masked:
        mask = torch.ones(B, N, dtype=torch.float64)
        mask[0, 12:] = 0
    gO = torch.randn(B, N, H * d, generator=g, dtype=torch.float64)
    gT = 0.1 * torch.randn(B, H, N, N, generator=g, dtype=torch.float64)
    gx = torch.randn(B, H, N, 3, generator=g, dtype=torch.float64)

    leaves = [t.clone().requires_grad_(True) for t in (C, lu, lv, V, x)]
    o, Tn, xc, O_avg = ort.compute_transport_output(leaves[3], None, leaves[1], leaves[2], leaves[0], eps,
                                                    x_res=leaves[4], mask=mask)
    ((o * gO).sum() + (Tn * gT).sum() + (xc * gx).sum()).backward()
    ref = dict(dC=leaves[0].grad, dlu=leaves[1].grad, dlv=leaves[2].grad, dV=leaves[3].grad, dx=leaves[4].grad)

    # the library's route: the gate is identity here (G = None), o = O_avg permuted and masked
    Tn = Tn.detach()
    dO_avg = gO.reshape(B, N, H, d).permute(0, 2, 1, 3)
    if mask is not None:
        dO_avg = dO_avg * mask[:, None, :, None]
    dT = dO_avg @ V.transpose(-1, -2) + gx @ x.transpose(-1, -2)[:, None] + gT
    dscore = Tn * (dT - (dT * Tn).sum(-1, keepdim=True))
    got = dict(dC=-dscore / eps[None, :, None, None], dlu=torch.zeros_like(lu), dlv=dscore.sum(-2),
               dV=Tn.transpose(-1, -2) @ dO_avg, dx=(Tn.transpose(-1, -2) @ gx).sum(1))
    for k in ref:
        scale = max(float(ref[k].abs().max()), 1.0)
        err = float((got[k] - ref[k]).abs().max())
        assert err <= 1e-5 * scale, (k, err, scale)  # the dropped rowmax term is ~1e-6 relative
