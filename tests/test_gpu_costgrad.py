"""Gradients of the shared cost parameters x_res, pos_weight and w_dist
(reference: sinkhorn_kernel.py:2366-2382 returns them beside dQ, dK, dV).

* the reference's own all-terms case (tests/golden/uot_full: d=8, per-head eps,
  lam=1, K=5, pos_bins, geometry, centroid with an upstream gradient), against
  the oracle's implicit adjoint at the same potentials (K=5 is not converged);
* a converged balanced case at d=32 against the oracle's unrolled gradient, the
  reference's own autograd semantics;
* bitwise reproducibility (the bin histogram is summed in fixed point).
Tolerance: relative error <= 5e-3 (the gradient bar of the parity criterion).
"""

import math
import os

import numpy as np
import pytest
import torch

from helpers import rel_err
from oracle import sinkhorn_oracle as orc

from deepfold.model.kernels.flash_sinkhorn_attn import flash_sinkhorn_attn

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
TOL = 5e-3


def _run(z, dev, K_iter, lam, r_0):
    t = lambda k: torch.tensor(z[k], device=dev)  # noqa: E731
    leaves = {k: t(k).float().requires_grad_(True) for k in ("in_Q", "in_K", "in_V", "in_G", "in_x", "in_pos_w",
                                                                "in_w_dist")}
    o, xc, _, _ = flash_sinkhorn_attn(leaves["in_Q"], leaves["in_K"], leaves["in_V"], leaves["in_G"], leaves["in_x"],
                                      leaves["in_pos_w"], t("in_bins"), t("in_eps"), leaves["in_w_dist"],
                                      t("in_log_mu"), t("in_log_nu"), K_iter=K_iter, lam=lam, r_0=r_0)
    ((o * t("in_dO")).sum() + (xc * t("in_dxc")).sum()).backward()
    torch.cuda.synchronize()
    names = dict(in_Q="dQ", in_K="dK", in_V="dV", in_G="dG", in_x="dx", in_pos_w="dpos", in_w_dist="dw")
    return {names[k]: v.grad.detach().cpu().numpy() for k, v in leaves.items()}


def _oracle(z, K_iter, lam, r_0, mode):
    _, gr = orc.flash_sinkhorn_attn(z["in_Q"], z["in_K"], z["in_V"], z["in_G"], z["in_x"], z["in_pos_w"],
                                    z["in_bins"], z["in_eps"], z["in_w_dist"], z["in_log_mu"], z["in_log_nu"],
                                    K_iter=K_iter, lam=lam, r_0=r_0, with_grad=True, dO_flat=z["in_dO"],
                                    dxc=z["in_dxc"], grad_mode=mode)
    return gr


def test_golden_all_terms_all_gradients_match_ift():
    zz = np.load(os.path.join(GOLD, "uot_full.npz"))
    z = {k: zz[k] for k in zz.files}
    K_iter, lam, r_0 = int(z["meta_K_iter"]), float(z["meta_lam"]), float(z["meta_r_0"])
    g = _run(z, torch.device("cuda"), K_iter, lam, r_0)
    ref = _oracle(z, K_iter, lam, r_0, "ift")
    for k in ("dQ", "dK", "dV", "dG", "dx", "dpos", "dw"):
        assert rel_err(g[k], ref[k]) <= TOL, f"{k}: {rel_err(g[k], ref[k]):.3e}"


def _synthetic(B, H, N, d, seed):
    r = np.random.default_rng(seed)
    f32 = np.float32
    z = dict(in_Q=r.standard_normal((B, H, N, d)), in_K=r.standard_normal((B, H, N, d)),
             in_V=r.standard_normal((B, H, N, d)), in_G=r.standard_normal((B, H, N, d)),
             in_x=3.0 * r.standard_normal((B, N, 3)), in_pos_w=0.5 * r.standard_normal((H, 68)),
             in_bins=r.integers(0, 68, (B, N, N)).astype(np.int32), in_eps=np.linspace(0.6, 1.4, H),
             in_w_dist=np.linspace(0.1, 0.9, H), in_log_mu=np.full((B, H, N), -math.log(N)),
             in_log_nu=np.full((B, H, N), -math.log(N)), in_dO=r.standard_normal((B, N, H * d)),
             in_dxc=r.standard_normal((B, H, N, 3)))
    # bf16-representable operands (the products are then exact on any path)
    for k in ("in_Q", "in_K", "in_V"):
        z[k] = torch.tensor(z[k]).to(torch.bfloat16).float().numpy()
    return {k: (v.astype(f32) if v.dtype.kind == "f" else v) for k, v in z.items()}


@pytest.mark.parametrize("N", [96, 200, 384])
def test_converged_all_gradients_match_unrolled(N):
    z = _synthetic(2, 4, N, 32, seed=N)
    g = _run(z, torch.device("cuda"), 80, math.inf, 10.0)
    ref = _oracle(z, 80, math.inf, 10.0, "unrolled")
    for k in ("dQ", "dK", "dV", "dG", "dx", "dpos", "dw"):
        assert rel_err(g[k], ref[k]) <= TOL, f"{k}: {rel_err(g[k], ref[k]):.3e}"


def test_shared_parameter_gradients_are_bitwise_reproducible():
    z = _synthetic(2, 4, 160, 32, seed=5)
    a = _run(z, torch.device("cuda"), 30, 1.0, 10.0)
    b = _run(z, torch.device("cuda"), 30, 1.0, 10.0)
    for k in ("dx", "dpos", "dw", "dQ", "dK"):
        assert np.array_equal(a[k], b[k]), k
