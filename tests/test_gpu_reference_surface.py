"""The reference's own operator tests, restated against this package on a B200.

The reference pins its drop-in surface with tests/test_flash_sinkhorn_batch.py
(batched == per-sample, unbatched shapes, B=1 == unbatched), tests/test_cg.py
(sinkhorn_solve early stop) and tests/test_sinkhorn_batch.py (padding
equivalence of the dense path).  Those files cannot travel to the GPU box, so
the same checks are written here, with the same shapes, seeds, argument values
and tolerances, and CPU tensors passed in as the reference passes them (the op
computes on the current CUDA device and returns CPU tensors).  On top of the
reference's self-consistency checks, every case is compared with the outputs of
the reference's own torch code stored in tests/golden/*.npz, or with the oracle.
"""

import math

import numpy as np
import pytest
import torch

from helpers import max_abs, rel_err
from oracle import sinkhorn_oracle as orc

from deepfold.model.kernels.flash_sinkhorn_attn import flash_sinkhorn_attn
from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve

pytestmark = pytest.mark.gpu

GOLDEN = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")


def flash_inputs(B, H, N, d, seed=42):
    """Seeded inputs in the form of tests/test_flash_sinkhorn_batch.py:6-23 of the
    reference: N(0,1) Q, K, V, G, x_res and pos_weight, random bins in [0, 68),
    per-head eps in four groups (0.5, 1, 2, 4), w_dist in [0, 0.5), log-softmax
    marginals -- drawn from one torch generator in that order."""
    g = torch.Generator().manual_seed(seed)
    Q, K, V, G = (torch.randn(B, H, N, d, generator=g) for _ in range(4))
    x = torch.randn(B, N, 3, generator=g)
    pos_w = torch.randn(H, 68, generator=g)
    bins = torch.randint(0, 68, (B, N, N), generator=g, dtype=torch.int32)
    q = H // 4
    eps = torch.tensor([0.5] * q + [1.0] * q + [2.0] * q + [4.0] * q, dtype=torch.float32)
    w = torch.rand(H, generator=g) * 0.5
    lmu = torch.log_softmax(torch.randn(B, H, N, generator=g), dim=-1)
    lnu = torch.log_softmax(torch.randn(B, H, N, generator=g), dim=-1)
    return Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu


def oracle_attn(args, K_iter, lam, r_0=10.0, mask=None):
    Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu = (a.numpy() for a in args)
    res, _ = orc.flash_sinkhorn_attn(Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu, K_iter=K_iter, lam=lam,
                                     r_0=r_0, mask=mask)
    return res


def test_batched_matches_per_sample():
    """tests/test_flash_sinkhorn_batch.py:29-107: B=2 H=4 N=16 d=8, K=3, lam=1."""
    B, H, N, d, K_iter = 2, 4, 16, 8, 3
    args = flash_inputs(B, H, N, d)
    o, xc, lu, lv = flash_sinkhorn_attn(*args, K_iter=K_iter, lam=1.0, r_0=10.0)
    assert o.shape == (B, N, H * d) and xc.shape == (B, H, N, 3)
    assert lu.shape == (B, H, N) and lv.shape == (B, H, N)
    assert o.device.type == "cpu"
    for b in range(B):
        Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu = args
        ob, xcb, lub, lvb = flash_sinkhorn_attn(Q[b], K[b], V[b], G[b], x[b], pos_w, bins[b], eps, w, lmu[b],
                                                lnu[b], K_iter=K_iter, lam=1.0, r_0=10.0)
        for got, want in ((o[b], ob), (xc[b], xcb), (lu[b], lub), (lv[b], lvb)):
            torch.testing.assert_close(got, want, atol=1e-4, rtol=1e-4)
    # and the values themselves: the oracle in float64 on the same inputs (the
    # kernels take fp32 operands through tf32 tensor-core products)
    ref = oracle_attn(args, K_iter, 1.0)
    assert max_abs(o.numpy(), ref.o_flat) <= 2e-3
    assert max_abs(xc.numpy(), ref.xc) <= 2e-3
    assert max_abs(lu.numpy(), ref.log_u) <= 2e-3
    assert max_abs(lv.numpy(), ref.log_v) <= 2e-3


def test_unbatched_shapes():
    """tests/test_flash_sinkhorn_batch.py:109-147: H=4 N=8 d=8, K=2, default lam."""
    args = [a[0] for a in flash_inputs(1, 4, 8, 8, seed=99)[:5]]
    Q, K, V, G, x = args
    _, _, _, _, _, pos_w, bins, eps, w, lmu, lnu = flash_inputs(1, 4, 8, 8, seed=99)
    o, xc, lu, lv = flash_sinkhorn_attn(Q, K, V, G, x, pos_w, bins[0], eps, w, lmu[0], lnu[0], K_iter=2)
    assert o.shape == (8, 4 * 8) and xc.shape == (4, 8, 3)
    assert lu.shape == (4, 8) and lv.shape == (4, 8)


def test_b1_matches_unbatched():
    """tests/test_flash_sinkhorn_batch.py:149-204: B=1 batched == unbatched at 1e-5."""
    Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu = flash_inputs(1, 4, 8, 8, seed=77)
    ub = flash_sinkhorn_attn(Q[0], K[0], V[0], G[0], x[0], pos_w, bins[0], eps, w, lmu[0], lnu[0], K_iter=3)
    bt = flash_sinkhorn_attn(Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu, K_iter=3)
    for a, b in zip(ub, bt):
        torch.testing.assert_close(a, b.squeeze(0), atol=1e-5, rtol=1e-5)


def _golden(name):
    z = np.load(f"{GOLDEN}/{name}.npz")
    return {k: z[k] for k in z.files}


def _leaves(z, keys, dev):
    return [torch.tensor(z[k], dtype=torch.float32, device=dev).requires_grad_(True) for k in keys]


@pytest.mark.parametrize("name,d", [("masked_varlen", 8), ("pure_balanced", 16)])
def test_golden_small_head_dims_forward_and_backward(name, d):
    """The reference's own outputs and autograd gradients (tests/golden) at head
    dims 8 and 16, balanced (lam = 1e6) and converged, so the IFT gradient equals
    the reference's unrolled one."""
    z = _golden(name)
    dev = torch.device("cuda")
    Q, K, V, G = _leaves(z, ("in_Q", "in_K", "in_V", "in_G"), dev)
    assert Q.shape[-1] == d
    mask = torch.tensor(z["in_mask"], device=dev) if "in_mask" in z else None
    eps = torch.tensor(z["in_eps"], device=dev)
    lmu = torch.tensor(z["in_log_mu"], device=dev)
    lnu = torch.tensor(z["in_log_nu"], device=dev)
    o, _, lu, lv = flash_sinkhorn_attn(Q, K, V, G, None, None, None, eps, None, lmu, lnu,
                                       K_iter=int(z["meta_K_iter"]), lam=float(z["meta_lam"]),
                                       r_0=float(z["meta_r_0"]), mask=mask)
    (o * torch.tensor(z["in_dO"], device=dev)).sum().backward()
    # fp32 operands: d = 8 runs as exact bf16 hi/lo products; d = 16 through tf32
    # tensor-core products (~2^-11 relative on the logits), as the reference's
    # own GPU path (tl.dot on fp32) does
    tol = 2e-3 if d <= 10 else 5e-3
    assert max_abs(o.detach().cpu().numpy(), z["out_o"]) <= tol
    assert max_abs(lu.cpu().numpy(), z["out_log_u"]) <= tol
    assert max_abs(lv.cpu().numpy(), z["out_log_v"]) <= tol
    for leaf, key in ((Q, "out_dQ"), (K, "out_dK"), (V, "out_dV"), (G, "out_dG")):
        assert rel_err(leaf.grad.cpu().numpy(), z[key]) <= 5e-3, key


def test_golden_uot_full_forward():
    """All cost terms at d = 8 (pos_bins, geometry, per-head eps, lam = 1, K = 5)
    against the reference's flash_sinkhorn_attn outputs (tests/golden/uot_full)."""
    z = _golden("uot_full")
    dev = torch.device("cuda")
    t = lambda k: torch.tensor(z[k], device=dev)  # noqa: E731
    o, xc, lu, lv = flash_sinkhorn_attn(t("in_Q"), t("in_K"), t("in_V"), t("in_G"), t("in_x"), t("in_pos_w"),
                                        t("in_bins"), t("in_eps"), t("in_w_dist"), t("in_log_mu"),
                                        t("in_log_nu"), K_iter=int(z["meta_K_iter"]), lam=float(z["meta_lam"]),
                                        r_0=float(z["meta_r_0"]))
    assert max_abs(o.cpu().numpy(), z["out_o"]) <= 2e-3
    assert max_abs(xc.cpu().numpy(), z["out_xc"]) <= 2e-3
    assert max_abs(lu.cpu().numpy(), z["out_log_u"]) <= 2e-3
    assert max_abs(lv.cpu().numpy(), z["out_log_v"]) <= 2e-3


def test_golden_uot_full_backward_matches_ift():
    """Same case, gradients of Q, K, V, G: K = 5 is not converged, so the kernels'
    implicit gradient is compared with the oracle's IFT adjoint at the same
    potentials (the reference's unrolled gradient differs there by design)."""
    z = _golden("uot_full")
    dev = torch.device("cuda")
    t = lambda k: torch.tensor(z[k], device=dev)  # noqa: E731
    Q, K, V, G = _leaves(z, ("in_Q", "in_K", "in_V", "in_G"), dev)
    o, _, _, _ = flash_sinkhorn_attn(Q, K, V, G, t("in_x"), t("in_pos_w"), t("in_bins"), t("in_eps"),
                                     t("in_w_dist"), t("in_log_mu"), t("in_log_nu"), K_iter=int(z["meta_K_iter"]),
                                     lam=float(z["meta_lam"]), r_0=float(z["meta_r_0"]))
    (o * t("in_dO")).sum().backward()
    _, gr = orc.flash_sinkhorn_attn(z["in_Q"], z["in_K"], z["in_V"], z["in_G"], z["in_x"], z["in_pos_w"],
                                    z["in_bins"], z["in_eps"], z["in_w_dist"], z["in_log_mu"], z["in_log_nu"],
                                    K_iter=int(z["meta_K_iter"]), lam=float(z["meta_lam"]),
                                    r_0=float(z["meta_r_0"]), with_grad=True, dO_flat=z["in_dO"], grad_mode="ift")
    for leaf, key in ((Q, "dQ"), (K, "dK"), (V, "dV"), (G, "dG")):
        assert rel_err(leaf.grad.cpu().numpy(), gr[key]) <= 5e-3, key


# ---------------------------------------------------------------- dense path


def test_sinkhorn_solve_early_stopping():
    """tests/test_cg.py:103-121: H=2 N=8, K=100, threshold 1e-3 vs none, atol 0.01."""
    torch.manual_seed(0)
    C = torch.randn(2, 8, 8).abs()
    lmu = torch.log_softmax(torch.randn(2, 8), dim=-1)
    lnu = torch.log_softmax(torch.randn(2, 8), dim=-1)
    eps = torch.tensor([1.0, 2.0])
    lu1, lv1 = sinkhorn_solve(C, lmu, lnu, eps, K=100, threshold=1e-3, check_every=2)
    lu2, lv2 = sinkhorn_solve(C, lmu, lnu, eps, K=100)
    assert lu1.device.type == "cpu"
    assert torch.allclose(lu1, lu2, atol=0.01)
    ref_u, ref_v = orc.sinkhorn_solve(C.numpy(), lmu.numpy(), lnu.numpy(), eps.numpy(), K=100)
    assert max_abs(lu2.numpy(), ref_u) <= 1e-4 and max_abs(lv2.numpy(), ref_v) <= 1e-4


def test_sinkhorn_solve_threshold_none_runs_all():
    """tests/test_cg.py:123-135: threshold=None is the default (all K iterations)."""
    torch.manual_seed(1)
    C = torch.randn(2, 4, 4).abs()
    lmu = torch.log_softmax(torch.randn(2, 4), dim=-1)
    lnu = torch.log_softmax(torch.randn(2, 4), dim=-1)
    eps = torch.tensor([1.0, 2.0])
    r1 = sinkhorn_solve(C, lmu, lnu, eps, K=3)
    r2 = sinkhorn_solve(C, lmu, lnu, eps, K=3, threshold=None)
    assert torch.equal(r1[0], r2[0]) and torch.equal(r1[1], r2[1])
    ref_u, ref_v = orc.sinkhorn_solve(C.numpy(), lmu.numpy(), lnu.numpy(), eps.numpy(), K=3)
    assert max_abs(r1[0].numpy(), ref_u) <= 1e-5 and max_abs(r1[1].numpy(), ref_v) <= 1e-5


@pytest.mark.parametrize("thr", [None, 1e-3])
def test_sinkhorn_solve_golden(thr):
    """The reference's sinkhorn_solve outputs (tests/golden/solve_early_stop): the
    full run at 1e-5; with the early stop, each problem here stops on its own
    L-inf test, so the results agree to the threshold."""
    z = _golden("solve_early_stop")
    dev = torch.device("cuda")
    t = lambda k: torch.tensor(z[k], device=dev)  # noqa: E731
    lu, lv = sinkhorn_solve(t("in_C"), t("in_log_mu"), t("in_log_nu"), t("in_eps"), lam=float(z["meta_lam"]),
                            K=int(z["meta_K_iter"]), threshold=thr)
    tag = "none" if thr is None else "1e-3"
    tol = 1e-5 if thr is None else 1e-3
    assert max_abs(lu.cpu().numpy(), z[f"out_log_u_{tag}"]) <= tol
    assert max_abs(lv.cpu().numpy(), z[f"out_log_v_{tag}"]) <= tol


def _dense_inputs(H, N, d, seed):
    """Dense-path inputs in the form of tests/test_sinkhorn_batch.py:8-19 of the
    reference: symmetric uniform cost, log-softmax marginals, eps = 0.1."""
    g = torch.Generator().manual_seed(seed)
    C = torch.rand(H, N, N, generator=g)
    C = C + C.transpose(-1, -2)
    lmu = torch.log_softmax(torch.randn(H, N, generator=g), dim=-1)
    lnu = torch.log_softmax(torch.randn(H, N, generator=g), dim=-1)
    eps = torch.full((H,), 0.1)
    V = torch.randn(H, N, d, generator=g)
    G = torch.randn(H, N, d, generator=g)
    x = torch.randn(N, 3, generator=g)
    return C, lmu, lnu, eps, V, G, x


def test_dense_unbatched_matches_batched():
    """tests/test_sinkhorn_batch.py:21-40: B=1 batched == unbatched at 1e-5."""
    C, lmu, lnu, eps, V, G, x = _dense_inputs(4, 8, 16, 42)
    ub = sinkhorn_solve(C, lmu, lnu, eps, K=10)
    bt = sinkhorn_solve(C[None], lmu[None], lnu[None], eps, K=10)
    assert bt[0].shape == (1, 4, 8)
    torch.testing.assert_close(ub[0], bt[0][0], atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(ub[1], bt[1][0], atol=1e-5, rtol=1e-5)
    o, T, xc = compute_transport_output(V, G, ub[0], ub[1], C, eps, x_res=x)
    assert o.shape == (8, 4 * 16) and T.shape == (4, 8, 8) and xc.shape == (4, 8, 3)
    # values: the oracle's transport on the same potentials
    for h in range(4):
        S = -C[h].double().numpy() / 0.1
        tr = orc.transport_problem(S, ub[0][h].double().numpy(), ub[1][h].double().numpy(), V[h].numpy(), x.numpy())
        sig = 1.0 / (1.0 + np.exp(-G[h].double().numpy()))
        assert max_abs(T[h].numpy(), tr.Tn) <= 1e-5
        # T_norm enters the tensor-core product O = T_norm V as tf32 (2^-11 relative), as
        # the reference's tl.dot does on the GPU
        assert max_abs(o.numpy().reshape(8, 4, 16)[:, h], sig * tr.O) <= 1e-3
        assert max_abs(xc[h].numpy(), tr.xc) <= 1e-4


def test_dense_padded_batch_matches_unpadded():
    """tests/test_sinkhorn_batch.py:43-200: a sample of N=5 padded to 8 beside a
    full one gives the unpadded sample's duals and outputs; padded duals and
    padded output rows are exactly 0."""
    H, N, n2, d, K_it = 4, 8, 5, 16, 10
    C1, lmu1, lnu1, eps, V1, G1, x1 = _dense_inputs(H, N, d, 1)
    C2r, lmu2r, lnu2r, _, V2r, G2r, x2r = _dense_inputs(H, n2, d, 2)
    C2 = torch.zeros(H, N, N)
    C2[:, :n2, :n2] = C2r
    lmu2 = torch.full((H, N), -1e9)
    lmu2[:, :n2] = lmu2r
    lnu2 = torch.full((H, N), -1e9)
    lnu2[:, :n2] = lnu2r
    V2 = torch.zeros(H, N, d)
    V2[:, :n2] = V2r
    G2 = torch.zeros(H, N, d)
    G2[:, :n2] = G2r
    x2 = torch.zeros(N, 3)
    x2[:n2] = x2r
    mask = torch.ones(2, N)
    mask[1, n2:] = 0
    C = torch.stack([C1, C2])
    lu, lv = sinkhorn_solve(C, torch.stack([lmu1, lmu2]), torch.stack([lnu1, lnu2]), eps, K=K_it, mask=mask)
    lu1, lv1 = sinkhorn_solve(C1, lmu1, lnu1, eps, K=K_it)
    lu2, lv2 = sinkhorn_solve(C2r, lmu2r, lnu2r, eps, K=K_it)
    torch.testing.assert_close(lu[0], lu1, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lu[1, :, :n2], lu2, atol=1e-5, rtol=1e-5)
    torch.testing.assert_close(lv[1, :, :n2], lv2, atol=1e-5, rtol=1e-5)
    assert torch.all(lu[1, :, n2:] == 0) and torch.all(lv[1, :, n2:] == 0)
    o, T, xc = compute_transport_output(torch.stack([V1, V2]), torch.stack([G1, G2]), lu, lv, C, eps,
                                        x_res=torch.stack([x1, x2]), mask=mask)
    o2, _, xc2 = compute_transport_output(V2r, G2r, lu2, lv2, C2r, eps, x_res=x2r)
    torch.testing.assert_close(o[1, :n2], o2, atol=1e-4, rtol=1e-4)
    torch.testing.assert_close(xc[1, :, :n2], xc2, atol=1e-4, rtol=1e-4)
    assert torch.all(o[1, n2:] == 0)
    assert torch.all(T[1, :, n2:] == 0)


def test_small_head_dim_grads_are_finite_and_match_oracle():
    """d = 8 (the reference tests' head dim) through the backward: zero-padded
    inside the library, gradients of Q, K, V against the oracle's IFT adjoint."""
    B, H, N, d = 2, 4, 16, 8
    Q, K, V, G, x, pos_w, bins, eps, w, lmu, lnu = flash_inputs(B, H, N, d, seed=5)
    dev = torch.device("cuda")
    leaves = [t.to(dev).requires_grad_(True) for t in (Q, K, V)]
    dO = torch.randn(B, N, H * d, generator=torch.Generator().manual_seed(6))
    o, _, _, _ = flash_sinkhorn_attn(*leaves, G.to(dev), x.to(dev), pos_w.to(dev), bins.to(dev), eps.to(dev),
                                     w.to(dev), lmu.to(dev), lnu.to(dev), K_iter=30, lam=math.inf)
    (o * dO.to(dev)).sum().backward()
    _, gr = orc.flash_sinkhorn_attn(Q.numpy(), K.numpy(), V.numpy(), G.numpy(), x.numpy(), pos_w.numpy(),
                                    bins.numpy(), eps.numpy(), w.numpy(), lmu.numpy(), lnu.numpy(), K_iter=30,
                                    lam=math.inf, with_grad=True, dO_flat=dO.numpy(), grad_mode="ift")
    for leaf, key in zip(leaves, ("dQ", "dK", "dV")):
        assert rel_err(leaf.grad.cpu().numpy(), gr[key]) <= 5e-3, key
