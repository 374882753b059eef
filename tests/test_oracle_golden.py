"""Pin the CPU oracle against golden vectors produced by the reference's own code.

The fixtures in tests/golden/ come from tests/golden/make_golden.py, which runs
the reference's torch implementation (sinkhorn_solve / compute_transport_output
/ flash_sinkhorn_attn and autograd through them).  The oracle is float64; the
reference ran in float32, so agreement is to float32 round-off.
"""

import os

import numpy as np
import pytest

from oracle import sinkhorn_oracle as orc

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def load(name):
    z = np.load(os.path.join(GOLD, name + ".npz"))
    inp = {k[3:]: z[k] for k in z.files if k.startswith("in_")}
    out = {k[4:]: z[k] for k in z.files if k.startswith("out_")}
    meta = {k[5:]: z[k].item() for k in z.files if k.startswith("meta_")}
    return inp, out, meta


def close(a, b, rtol, atol, what):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    err = np.max(np.abs(a - b) / (atol + rtol * np.abs(b)))
    assert err <= 1.0, f"{what}: max scaled error {err:.3g}"


def rel(a, b):
    return float(np.max(np.abs(a - b)) / max(np.max(np.abs(b)), 1e-30))


def test_pure_balanced():
    inp, out, meta = load("pure_balanced")
    res, gr = orc.flash_sinkhorn_attn(
        inp["Q"], inp["K"], inp["V"], inp["G"], None, None, None, inp["eps"], None,
        inp["log_mu"], inp["log_nu"], K_iter=meta["K_iter"], lam=meta["lam"],
        with_grad=True, dO_flat=inp["dO"])
    close(res.o_flat, out["o"], 1e-4, 1e-5, "o")
    close(res.log_u, out["log_u"], 1e-4, 1e-4, "log_u")
    close(res.log_v, out["log_v"], 1e-4, 1e-4, "log_v")
    for k in ("dQ", "dK", "dV", "dG"):
        assert rel(gr[k], out[k]) < 2e-4, k


@pytest.mark.parametrize("tag,lam", [("bal", 1e6), ("uot", 1.0)])
def test_config0(tag, lam):
    inp, out, meta = load("config0")
    B, H, N, d = inp["Q"].shape
    res, gr = orc.flash_sinkhorn_attn(
        inp["Q"], inp["K"], inp["V"], None, None, None, None, inp["eps"], None,
        inp["log_mu"], inp["log_nu"], K_iter=meta["K_iter"], lam=lam,
        with_grad=True, dO_flat=inp["dO"])
    close(res.o_flat, out["o_" + tag], 1e-4, 1e-5, "o")
    close(res.log_u, out["log_u_" + tag], 1e-4, 1e-4, "log_u")
    close(res.log_v, out["log_v_" + tag], 1e-4, 1e-4, "log_v")
    for k in ("dQ", "dK", "dV"):
        assert rel(gr[k], out[k + "_" + tag]) < 2e-4, k


def test_uot_full_features():
    inp, out, meta = load("uot_full")
    res, gr = orc.flash_sinkhorn_attn(
        inp["Q"], inp["K"], inp["V"], inp["G"], inp["x"], inp["pos_w"], inp["bins"],
        inp["eps"], inp["w_dist"], inp["log_mu"], inp["log_nu"], K_iter=meta["K_iter"],
        lam=meta["lam"], r_0=meta["r_0"], with_grad=True, dO_flat=inp["dO"], dxc=inp["dxc"])
    # forward pinned against the reference's flash_sinkhorn_attn (its distance has
    # no 1e-8 under the root, a ~1e-5 perturbation on the diagonal)
    close(res.o_flat, out["o"], 1e-4, 1e-4, "o")
    close(res.xc, out["xc"], 1e-4, 1e-4, "x_centroid")
    close(res.log_u, out["log_u"], 1e-4, 1e-4, "log_u")
    close(res.log_v, out["log_v"], 1e-4, 1e-4, "log_v")
    close(res.o_flat, out["o_dense"], 1e-4, 1e-5, "o vs dense")
    for k in ("dQ", "dK", "dV", "dG", "dx", "dpos", "dw"):
        assert rel(gr[k], out[k]) < 5e-4, k


def test_masked_varlen():
    inp, out, meta = load("masked_varlen")
    res, gr = orc.flash_sinkhorn_attn(
        inp["Q"], inp["K"], inp["V"], inp["G"], None, None, None, inp["eps"], None,
        inp["log_mu"], inp["log_nu"], K_iter=meta["K_iter"], lam=meta["lam"],
        mask=inp["mask"], with_grad=True, dO_flat=inp["dO"])
    close(res.o_flat, out["o"], 1e-4, 1e-5, "o")
    close(res.log_u, out["log_u"], 1e-4, 1e-4, "log_u")
    close(res.log_v, out["log_v"], 1e-4, 1e-4, "log_v")
    for k in ("dQ", "dK", "dV", "dG"):
        assert rel(gr[k], out[k]) < 2e-4, k
    # padded rows/cols: exact zeros, as tests/test_sinkhorn_batch.py:94-112 require
    m = inp["mask"]
    assert np.all(res.log_u[1][:, m[1] == 0] == 0) and np.all(res.log_v[1][:, m[1] == 0] == 0)
    assert np.all(res.o_flat[1][m[1] == 0] == 0)


@pytest.mark.parametrize("key,thr", [("none", None), ("1e-3", 1e-3)])
def test_solve_early_stop(key, thr):
    inp, out, meta = load("solve_early_stop")
    lu, lv = orc.sinkhorn_solve(inp["C"], inp["log_mu"], inp["log_nu"], inp["eps"],
                                lam=meta["lam"], K=meta["K_iter"], threshold=thr, check_every=2)
    close(lu, out["log_u_" + key], 1e-4, 1e-4, "log_u")
    close(lv, out["log_v_" + key], 1e-4, 1e-4, "log_v")


def test_ift_equals_unrolled_at_fixed_point():
    """The CG/IFT adjoint the CUDA backward solves equals the unrolled gradient once converged."""
    inp, out, meta = load("pure_balanced")
    kw = dict(K_iter=300, lam=float("inf"), with_grad=True, dO_flat=inp["dO"])
    args = (inp["Q"], inp["K"], inp["V"], inp["G"], None, None, None, inp["eps"], None,
            inp["log_mu"], inp["log_nu"])
    _, gu = orc.flash_sinkhorn_attn(*args, **kw)
    _, gi = orc.flash_sinkhorn_attn(*args, grad_mode="ift", **kw)
    for k in ("dQ", "dK", "dV", "dG", "dlog_mu", "dlog_nu"):
        assert rel(gi[k], gu[k]) < 1e-6, k


def test_ift_equals_unrolled_uot_masked():
    inp, out, meta = load("masked_varlen")
    kw = dict(K_iter=400, lam=1.0, mask=inp["mask"], with_grad=True, dO_flat=inp["dO"])
    args = (inp["Q"], inp["K"], inp["V"], inp["G"], None, None, None, inp["eps"], None,
            inp["log_mu"], inp["log_nu"])
    _, gu = orc.flash_sinkhorn_attn(*args, **kw)
    _, gi = orc.flash_sinkhorn_attn(*args, grad_mode="ift", **kw)
    for k in ("dQ", "dK", "dV", "dlog_mu", "dlog_nu"):
        assert rel(gi[k], gu[k]) < 1e-6, k
