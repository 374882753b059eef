"""Gradients of the dense-cost entry points (sinkhorn_solve, compute_transport_output)
against torch autograd through the reference's own computation restated in
oracle/sinkhorn_torch.py, in float64 -- what the reference's users get from
autograd (src/deepfold/model/sinkhorn.py:30-36) and what its gradient test
exercises (tests/test_primitives.py:152-164).

Bar: every gradient within 2e-3 of its largest magnitude (the library computes
in fp32 with ex2.approx exponentials; the oracle in float64)."""

import math

import pytest
import torch

from oracle import sinkhorn_torch as ort

from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve

from test_gpu_dense_stream import dense_case

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")
TOL = 2e-3


def close(got, ref, what):
    got, ref = got.detach().cpu().double(), ref.detach().cpu().double()
    scale = max(float(ref.abs().max()), 1e-12)
    err = float((got - ref).abs().max())
    assert err <= TOL * scale, f"{what}: max err {err:.3e} vs scale {scale:.3e}"


def leaves(*ts, dev=None, dtype=None):
    out = []
    for t in ts:
        if t is None:
            out.append(None)
            continue
        t = t.detach().clone()
        if dtype is not None:
            t = t.to(dtype)
        if dev is not None:
            t = t.to(dev)
        out.append(t.requires_grad_(True))
    return out


def solve_grads(fn, C, lmu, lnu, lvi, eps, lam, K, mask, gu, gv, threshold=None, dev=None, dtype=None):
    Cl, mul, nul, lvl = leaves(C, lmu, lnu, lvi, dev=dev, dtype=dtype)
    mv = lambda t: None if t is None else t.to(dev if dev is not None else t.device, dtype or t.dtype)  # noqa: E731
    lu, lv = fn(Cl, mul, nul, mv(eps), lam=lam, K=K, log_v_init=lvl, threshold=threshold, mask=mv(mask))
    loss = (lu * mv(gu)).sum() + (lv * mv(gv)).sum()
    loss.backward()
    return lu, lv, Cl.grad, mul.grad, nul.grad, lvl.grad


@pytest.mark.parametrize("N", [520, 515])          # 16-byte rows (vector loads) and ragged rows
@pytest.mark.parametrize("lam", [1.0, math.inf])
def test_solve_gradients_match_unrolled_autograd(N, lam):
    C, lmu, lnu, eps, _, _, _, mask = dense_case(2, 3, N, 8, seed=N + 7, lengths=[N, 401])
    g = torch.Generator().manual_seed(N)
    gu, gv, lvi = (torch.randn(2, 3, N, generator=g) for _ in range(3))
    lvi = 0.3 * lvi
    ours = solve_grads(sinkhorn_solve, C, lmu, lnu, lvi, eps, lam, 12, mask, gu, gv, dev=DEV)
    ref = solve_grads(ort.sinkhorn_solve, C, lmu, lnu, lvi, eps, lam, 12, mask, gu, gv, dtype=torch.float64)
    for what, a, b in zip(("log_u", "log_v", "dC", "dlog_mu", "dlog_nu", "dlog_v_init"), ours, ref):
        close(a, b, what)
    # padded rows / columns get no gradient
    assert float(ours[2][1, :, 401:, :].abs().max()) == 0.0
    assert float(ours[2][1, :, :, 401:].abs().max()) == 0.0
    assert float(ours[3][1, :, 401:].abs().max()) == 0.0


def test_solve_gradient_reference_unit_case_on_cpu_tensors():
    """The reference's test_unrolled_gradient case (H=2, N=5, randn cost, K=7,
    loss sum(log_u^2 + log_v^2)) on unbatched CPU tensors."""
    g = torch.Generator().manual_seed(0)
    C = torch.randn(2, 5, 5, generator=g)
    lmu = torch.log_softmax(torch.randn(2, 5, generator=g), dim=-1)
    lnu = torch.log_softmax(torch.randn(2, 5, generator=g), dim=-1)
    eps = torch.tensor([1.0, 2.0])
    grads = []
    for fn, dt in ((sinkhorn_solve, torch.float32), (ort.sinkhorn_solve, torch.float64)):
        Cl = C.clone().to(dt).requires_grad_(True)
        if fn is ort.sinkhorn_solve:
            lu, lv = fn(Cl[None], lmu.to(dt)[None], lnu.to(dt)[None], eps.to(dt), K=7)
        else:
            lu, lv = fn(Cl, lmu, lnu, eps, K=7)
        (lu ** 2 + lv ** 2).sum().backward()
        assert Cl.grad is not None and torch.isfinite(Cl.grad).all()
        grads.append(Cl.grad)
    assert grads[0].device.type == "cpu"
    close(grads[0], grads[1], "dC")


def test_solve_gradients_with_early_stop_follow_the_reference_stop():
    """threshold set: the batch-wide test every check_every iterations stops both
    at the same iteration, and the gradients are those of the iterations run."""
    C, lmu, lnu, eps, _, _, _, mask = dense_case(1, 2, 256, 8, seed=5, lengths=[256])
    g = torch.Generator().manual_seed(1)
    gu, gv, lvi = (torch.randn(1, 2, 256, generator=g) for _ in range(3))
    for thr in (1e-2, 1e-4):
        ours = solve_grads(sinkhorn_solve, C, lmu, lnu, 0 * lvi, eps, 1.0, 40, None, gu, gv, threshold=thr, dev=DEV)
        ref = solve_grads(ort.sinkhorn_solve, C, lmu, lnu, 0 * lvi, eps, 1.0, 40, None, gu, gv, threshold=thr,
                          dtype=torch.float64)
        for what, a, b in zip(("log_u", "log_v", "dC", "dlog_mu", "dlog_nu"), ours, ref):
            close(a, b, f"{what} (threshold {thr})")


def transport_grads(fn, V, G, lu, lv, C, eps, x, mask, go, gT, gx, dev=None, dtype=None):
    Vl, lul, lvl, Cl, xl = leaves(V, lu, lv, C, x, dev=dev, dtype=dtype)
    mv = lambda t: None if t is None else t.to(dev if dev is not None else t.device, dtype or t.dtype)  # noqa: E731
    out = fn(Vl, mv(G), lul, lvl, Cl, mv(eps), x_res=xl, mask=mv(mask))
    o, T, xc = out[0], out[1], out[2]
    loss = (o * mv(go)).sum() + (T * mv(gT)).sum() + (xc * mv(gx)).sum()
    loss.backward()
    return o, T, xc, Vl.grad, lvl.grad, Cl.grad, xl.grad, lul.grad


@pytest.mark.parametrize("N,d", [(600, 48), (515, 100)])
def test_transport_gradients_match_autograd(N, d):
    B, H = 2, 2
    C, lmu, lnu, eps, V, G, x, mask = dense_case(B, H, N, d, seed=N + d, lengths=[N, 333])
    ru, rv = ort.sinkhorn_solve(C.double(), lmu.double(), lnu.double(), eps.double(), K=8, mask=mask.double())
    g = torch.Generator().manual_seed(d)
    go = torch.randn(B, N, H * d, generator=g)
    gT = 0.1 * torch.randn(B, H, N, N, generator=g)
    gx = torch.randn(B, H, N, 3, generator=g)
    ours = transport_grads(compute_transport_output, V, G, ru.float(), rv.float(), C, eps, x, mask, go, gT, gx,
                           dev=DEV)
    ref = transport_grads(ort.compute_transport_output, V, G, ru, rv, C, eps, x, mask, go, gT, gx,
                          dtype=torch.float64)
    for what, a, b in zip(("o", "T_norm", "x_centroid", "dV", "dlog_v", "dC", "dx_res"), ours, ref):
        close(a, b, what)
    # log_u cancels in score - rowmax: its gradient is zero (the oracle's is rounding noise)
    assert float(ours[7].abs().max()) == 0.0
    assert float(ref[7].abs().max()) <= 1e-6 * float(ref[4].abs().max())


def test_solve_then_transport_end_to_end():
    """Cost -> sinkhorn_solve -> compute_transport_output -> loss, gradients to
    the cost through both calls (the reference's dense pipeline)."""
    C, lmu, lnu, eps, V, G, x, mask = dense_case(1, 2, 400, 32, seed=3, lengths=[400])
    g = torch.Generator().manual_seed(2)
    go = torch.randn(1, 400, 64, generator=g)
    res = []
    for solve, trans, dev, dt in ((sinkhorn_solve, compute_transport_output, DEV, torch.float32),
                                  (ort.sinkhorn_solve, ort.compute_transport_output, torch.device("cpu"),
                                   torch.float64)):
        Cl, Vl = leaves(C, V, dev=dev, dtype=dt)
        mv = lambda t: t.to(dev, dt)  # noqa: E731
        lu, lv = solve(Cl, mv(lmu), mv(lnu), mv(eps), K=10)
        o = trans(Vl, mv(G), lu, lv, Cl, mv(eps))[0]
        (o * mv(go)).sum().backward()
        res.append((o, Cl.grad, Vl.grad))
    for what, a, b in zip(("o", "dC", "dV"), res[0], res[1]):
        close(a, b, what)
