"""Gradients of the dense-cost entry points (sinkhorn_solve, compute_transport_output)
against torch autograd through the reference's own computation restated in
oracle/sinkhorn_torch.py, in float64 -- what the reference's users get from
autograd (src/deepfold/model/sinkhorn.py:30-36) and what its gradient test
exercises (tests/test_primitives.py:152-164).

Bar: every gradient within 2e-3 of its largest magnitude (the library computes
in fp32 with ex2.approx exponentials; the oracle in float64)."""

import math

import numpy as np
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


def _pass_ranges(C, lmu, lnu, lvi, eps, K, mask):
    """Per head, the two quantities that pick the factored or the exact cost
    pass (log2 units, valid points): the largest row range over iterations
    1..K of u_i plus the largest column range of v_i / kappa - log_nu, and the
    same for u_i / kappa - log_mu and v_i-1 (iterations 0..K-1)."""
    kap = (1.0 / (1.0 + eps.double()))[None, :, None]
    us, vs = [], [lvi.double()]
    for k in range(1, K + 1):
        u, v = ort.sinkhorn_solve(C.double(), lmu.double(), lnu.double(), eps.double(), K=k,
                                  log_v_init=lvi.double(), mask=mask.double())
        us.append(u)
        vs.append(v)
    valid = mask[:, None, :].bool().expand_as(us[0])
    # padded points are zeroed in the returned potentials: only valid ones count

    def rng(xs):
        xs = torch.stack(xs) * 1.4427
        r = torch.where(valid, xs.max(0).values - xs.min(0).values, torch.zeros_like(xs[0]))
        return [float(r[:, h].max()) for h in range(C.shape[1])]
    ru = rng(us)
    rvc = rng([v / kap - lnu.double() for v in vs[1:]])
    rur = rng([u / kap - lmu.double() for u in us])
    rvr = rng(vs[:-1])
    return [(ru[h] + rvc[h], rur[h] + rvr[h]) for h in range(C.shape[1])]


@pytest.mark.parametrize("mode", ["auto", "exact"])
def test_solve_gradients_exact_and_factored_cost_pass_in_one_call(mode, monkeypatch):
    """The cost gradient is formed by a factored (rank-2K) pass while a problem's
    row and column potentials stay within a 2^64 range over the iterations, else
    by the exact per-term pass.  eps = 0.02 moves the potentials far (the exact
    pass), eps = 1 does not (the factored pass): one call runs both.  (The
    ranges are computed from the float64 oracle's iterates.)  With
    DFS_DENSE_DC=exact every problem takes the exact pass.  Each head is
    checked on its own scale."""
    if mode == "exact":
        monkeypatch.setenv("DFS_DENSE_DC", "exact")
    N = 260
    C, lmu, lnu, _, _, _, _, mask = dense_case(2, 2, N, 8, seed=11, lengths=[N, 200])
    eps = torch.tensor([0.02, 1.0])
    g = torch.Generator().manual_seed(5)
    gu, gv, lvi = (torch.randn(2, 2, N, generator=g) for _ in range(3))
    lvi = 0.1 * lvi
    lvi[:, 0] *= 500.0  # head 0 starts far from its fixed point
    ranges = _pass_ranges(C, lmu, lnu, lvi, eps, 6, mask)
    assert max(ranges[0]) > 64 and max(ranges[1]) < 64, ranges
    ours = solve_grads(sinkhorn_solve, C, lmu, lnu, lvi, eps, 1.0, 6, mask, gu, gv, dev=DEV)
    ref = solve_grads(ort.sinkhorn_solve, C, lmu, lnu, lvi, eps, 1.0, 6, mask, gu, gv, dtype=torch.float64)
    for hd in range(2):
        for what, a, b in zip(("log_u", "log_v", "dC", "dlog_mu", "dlog_nu", "dlog_v_init"), ours, ref):
            close(a[:, hd], b[:, hd], f"{what} head {hd}")
    assert float(ours[2][1, :, 200:, :].abs().max()) == 0.0


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


@pytest.mark.parametrize("name", ["pure_balanced", "masked_varlen", "uot_full"])
def test_dense_gradients_match_the_reference_autograd_goldens(name):
    """The golden vectors hold the reference's own autograd through its cost,
    sinkhorn_solve and compute_transport_output (tests/golden/make_golden.py):
    the same loss through this library's dense entry points on the GPU (the
    cost itself formed by torch ops, as the reference's user forms it) gives
    the reference's outputs and the gradients of every input, including the
    position table, the geometry weight and the coordinates (uot_full)."""
    from test_oracle_torch import load

    inp, out, meta = load(name)
    f32 = lambda k: inp[k].to(DEV, torch.float32)  # noqa: E731
    leaf = lambda k: f32(k).requires_grad_(True)  # noqa: E731
    Q, K, V, G = leaf("Q"), leaf("K"), leaf("V"), leaf("G")
    full = name == "uot_full"
    x = leaf("x") if full else None
    pos = leaf("pos_w") if full else None
    w = leaf("w_dist") if full else None
    bins = inp["bins"].to(DEV) if full else None
    mask = f32("mask") if "mask" in inp else None
    eps = f32("eps")
    C = ort.cost(Q, K, x, pos, bins, w, float(meta["r_0"]))
    lu, lv = sinkhorn_solve(C, f32("log_mu"), f32("log_nu"), eps, lam=float(meta["lam"]), K=int(meta["K_iter"]),
                            mask=mask)
    o, _, xc = compute_transport_output(V, G, lu, lv, C, eps, x_res=x, mask=mask)
    loss = (o * f32("dO")).sum()
    if full:
        loss = loss + (xc * f32("dxc")).sum()
    loss.backward()

    def rel(a, b):
        return float(np.max(np.abs(a.detach().cpu().double().numpy() - b)) / max(np.max(np.abs(b)), 1e-30))
    assert rel(o, out["o_dense" if full else "o"]) < 1e-3
    if not full:  # uot_full's potentials are the flash path's (unconverged at K = 5)
        assert float(np.max(np.abs(lu.detach().cpu().numpy() - out["log_u"]))) < 1e-3
        assert float(np.max(np.abs(lv.detach().cpu().numpy() - out["log_v"]))) < 1e-3
    grads = dict(dQ=Q.grad, dK=K.grad, dV=V.grad, dG=G.grad)
    if full:
        grads.update(dx=x.grad, dpos=pos.grad, dw=w.grad)
    for k, g in grads.items():
        assert rel(g, out[k]) < TOL, (k, rel(g, out[k]))
