"""Pin the torch restatement of the reference's CPU path (oracle/sinkhorn_torch.py)
against the golden vectors produced by the reference's own code, and against the
float64 numpy oracle.  These two restatements are the checkers of the parity
tests and the timed CPU baseline of bench.py."""

import math
import os

import numpy as np
import pytest
import torch

from oracle import sinkhorn_oracle as orc
from oracle import sinkhorn_torch as ort

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    z = np.load(os.path.join(GOLD, name + ".npz"))
    t = lambda a: torch.tensor(a, dtype=torch.float64) if a.dtype.kind == "f" else torch.tensor(a)  # noqa: E731
    inp = {k[3:]: t(z[k]) for k in z.files if k.startswith("in_")}
    out = {k[4:]: z[k] for k in z.files if k.startswith("out_")}
    meta = {k[5:]: z[k].item() for k in z.files if k.startswith("meta_")}
    return inp, out, meta


def rel(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def _grads(inp, meta, lam, G=None, x=None, pos=None, bins=None, w=None, mask=None, dxc=None):
    leaves = {k: inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V")}
    G = None if G is None else G.clone().requires_grad_(True)
    o, O_avg, xc, lu, lv = ort.attn(leaves["Q"], leaves["K"], leaves["V"], inp["eps"], inp["log_mu"],
                                    inp["log_nu"], int(meta["K_iter"]), lam, G=G, x_res=x, pos_weight=pos,
                                    bins=bins, w_dist=w, r_0=float(meta.get("r_0", 10.0)), mask=mask)
    loss = (o * inp["dO"]).sum()
    if dxc is not None:
        loss = loss + (xc * dxc).sum()
    loss.backward()
    return o, xc, lu, lv, leaves, G


@pytest.mark.parametrize("name", ["pure_balanced", "masked_varlen"])
def test_golden_dense_forward_and_autograd(name):
    inp, out, meta = load(name)
    o, _, lu, lv, leaves, G = _grads(inp, meta, meta["lam"], G=inp["G"], mask=inp.get("mask"))
    assert rel(o.detach(), out["o"]) < 1e-4
    assert np.max(np.abs(lu.detach().numpy() - out["log_u"])) < 1e-4
    assert np.max(np.abs(lv.detach().numpy() - out["log_v"])) < 1e-4
    for k in ("Q", "K", "V"):
        assert rel(leaves[k].grad, out["d" + k]) < 2e-4, k
    assert rel(G.grad, out["dG"]) < 2e-4


def test_golden_all_cost_terms():
    inp, out, meta = load("uot_full")
    o, xc, lu, lv, leaves, G = _grads(inp, meta, meta["lam"], G=inp["G"], x=inp["x"], pos=inp["pos_w"],
                                      bins=inp["bins"], w=inp["w_dist"], dxc=inp["dxc"])
    assert rel(o.detach(), out["o_dense"]) < 1e-4
    assert rel(xc.detach(), out["xc"]) < 1e-4
    for k in ("Q", "K", "V"):
        assert rel(leaves[k].grad, out["d" + k]) < 2e-4, k


@pytest.mark.parametrize("tag,lam", [("bal", 1e6), ("uot", 1.0)])
def test_golden_config0(tag, lam):
    inp, out, meta = load("config0")
    o, _, lu, lv, leaves, _ = _grads(inp, meta, lam)
    assert rel(o.detach(), out["o_" + tag]) < 1e-4
    for k in ("Q", "K", "V"):
        assert rel(leaves[k].grad, out[f"d{k}_{tag}"]) < 2e-4, k


@pytest.mark.parametrize("thr", [None, 1e-3])
def test_golden_sinkhorn_solve(thr):
    inp, out, meta = load("solve_early_stop")
    lu, lv = ort.sinkhorn_solve(inp["C"], inp["log_mu"], inp["log_nu"], inp["eps"], lam=meta["lam"],
                                K=int(meta["K_iter"]), threshold=thr)
    tag = "none" if thr is None else "1e-3"
    assert np.max(np.abs(lu.numpy() - out[f"log_u_{tag}"])) < 1e-5
    assert np.max(np.abs(lv.numpy() - out[f"log_v_{tag}"])) < 1e-5


def test_agrees_with_numpy_oracle_balanced_inf():
    g = torch.Generator().manual_seed(3)
    B, H, N, d, K_it = 1, 2, 40, 16, 30
    Q, K, V = (torch.randn(B, H, N, d, generator=g, dtype=torch.float64) for _ in range(3))
    dO = torch.randn(B, H, N, d, generator=g, dtype=torch.float64)
    eps = torch.tensor([1.0, 0.7], dtype=torch.float64)
    lm = torch.full((B, H, N), -math.log(N), dtype=torch.float64)
    O, lu, lv, dQ, dK, dV = ort.attn_fwd_bwd(Q, K, V, eps, lm, lm, K_it, math.inf, dO, dtype=torch.float64)
    dO_flat = dO.numpy().transpose(0, 2, 1, 3).reshape(B, N, H * d)
    res, gr = orc.flash_sinkhorn_attn(Q.numpy(), K.numpy(), V.numpy(), None, None, None, None, eps.numpy(), None,
                                      lm.numpy(), lm.numpy(), K_iter=K_it, lam=math.inf, with_grad=True,
                                      dO_flat=dO_flat)
    assert rel(O, res.O_avg) < 1e-10
    assert rel(dQ, gr["dQ"]) < 1e-9 and rel(dK, gr["dK"]) < 1e-9 and rel(dV, gr["dV"]) < 1e-9
    r, c = ort.marginal_residuals(Q, K, eps, lu, lv, lm, lm)
    assert r < 1e-6 and c < 1e-6


@pytest.mark.parametrize("lam,masked", [(math.inf, False), (1.0, True)])
def test_problem_ift_matches_numpy_oracle(lam, masked):
    """The torch float64 IFT checker (used at N = 8192) against the numpy oracle's
    IFT adjoint on a small problem, balanced and unbalanced with padding."""
    g = torch.Generator().manual_seed(11)
    N, d, eps, K_it = 48, 16, 0.7, 60
    q, k, v, dO = (torch.randn(N, d, generator=g, dtype=torch.float64) for _ in range(4))
    mask = torch.ones(N, dtype=torch.float64)
    if masked:
        mask[37:] = 0
    cnt = float(mask.sum())
    a = torch.where(mask > 0, torch.log_softmax(torch.randn(N, generator=g, dtype=torch.float64)
                                                .masked_fill(mask == 0, -1e30), 0), torch.full((N,), -1e9,
                                                                                         dtype=torch.float64))
    b = torch.where(mask > 0, torch.full((N,), -math.log(cnt), dtype=torch.float64),
                    torch.full((N,), -1e9, dtype=torch.float64))
    out = ort.problem_fwd_bwd_ift(q, k, v, dO, eps, a, b, K_it, lam, mask=mask if masked else None)
    res, gr = orc.flash_sinkhorn_attn(q[None, None].numpy(), k[None, None].numpy(), v[None, None].numpy(), None,
                                      None, None, None, np.array([eps]), None, a[None, None].numpy(),
                                      b[None, None].numpy(), K_iter=K_it, lam=lam,
                                      mask=mask[None].numpy() if masked else None, with_grad=True,
                                      dO_flat=dO[None].numpy(), grad_mode="ift")
    assert rel(out["O"], res.O_avg[0, 0]) < 1e-10
    assert np.max(np.abs(out["log_u"].numpy() - res.log_u[0, 0])) < 1e-9
    for key in ("dQ", "dK", "dV"):
        assert rel(out[key], gr[key][0, 0]) < 1e-8, key


def test_golden_compute_bins():
    z = np.load(os.path.join(GOLD, "position_bins.npz"))
    ch, gx, bd = (torch.tensor(z["in_" + k]) for k in ("chain_id", "global_idx", "bond"))
    assert np.array_equal(ort.compute_bins(ch, gx, bd).numpy(), z["out_bins"])
    assert np.array_equal(ort.compute_bins(ch[0], gx[0], bd[0]).numpy(), z["out_bins_unbatched"])
