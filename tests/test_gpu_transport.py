"""Balanced transport of the trunk block on the GPU: balanced_sinkhorn_transport
and balanced_sinkhorn_transport_dual (reference: flash_sinkhorn_transport.py:376,
519) against the reference's own device path (tests/golden/balanced_device.npz:
its Triton kernels, forward and unrolled backward) and against the float64
oracle (oracle/transport_torch.py, pinned to those vectors) on bf16 inputs, on
the cluster-resident (N <= 384) and streamed (N > 384) kernels.

Tolerances: the parity bar of the operator -- outputs max-abs error <= 2e-3,
gradients relative error (norm of the difference over the norm of the
reference) <= 5e-3.  fp32 inputs run their Q K^T on tf32 tensor cores (the
reference's device path does the same with tl.dot); bf16 inputs give exact
products.  T_norm V runs with T_norm in bf16 (~4e-4 relative on h_centroid),
the backward's products of the fp32 adjoint dS on tf32 (~2e-3 relative).  The cosine
cost converges in about 10 iterations, so at K_iter = 20 the implicit
gradient of the op and the reference's unrolled one agree to rounding.
"""

import os

import numpy as np
import pytest
import torch
import torch.nn.functional as F

from helpers import rel_err
from oracle import transport_torch as tt

from deepfold.model.kernels.flash_sinkhorn_transport import (balanced_sinkhorn_transport,
                                                             balanced_sinkhorn_transport_dual)

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")
GRADS = ("Q", "K", "x", "V", "alpha", "r_h")


def _golden():
    z = np.load(os.path.join(GOLD, "balanced_device.npz"))
    return {k[3:]: torch.tensor(z[k]) for k in z.files if k.startswith("in_")}, \
        {k[4:]: z[k] for k in z.files if k.startswith("out_")}


def _run(inp, dual=True, K_iter=20, dtype=None, cg_opts=None):
    """The op on the GPU with leaves for Q, K, x, V, alpha, r_h; returns outputs
    and gradients of sum(gxc * xc) (+ sum(ghc * hc)) as CPU float64 arrays."""
    dev = torch.device("cuda")
    cast = (lambda t: t.to(dtype)) if dtype is not None else (lambda t: t)
    lv = {k: cast(inp[k]).to(dev).requires_grad_(True) for k in ("Q", "K", "V")}
    lv.update({k: inp[k].float().to(dev).requires_grad_(True) for k in ("x", "alpha", "r_h")})
    mask = inp["mask"].to(dev) if inp.get("mask") is not None else None
    eps = inp["eps"].float().to(dev)
    if dual:
        xc, hc = balanced_sinkhorn_transport_dual(lv["Q"], lv["K"], lv["x"], lv["V"], eps, lv["alpha"], lv["r_h"],
                                                  K_iter=K_iter, mask=mask, cg_opts=cg_opts)
        loss = (xc * inp["gxc"].to(dev)).sum() + (hc * inp["ghc"].to(dev)).sum()
    else:
        xc = balanced_sinkhorn_transport(lv["Q"], lv["K"], lv["x"], eps, lv["alpha"], lv["r_h"], K_iter=K_iter,
                                         mask=mask, cg_opts=cg_opts)
        hc = None
        loss = (xc * inp["gxc"].to(dev)).sum()
    loss.backward()
    torch.cuda.synchronize()
    out = {"xc": xc.detach().double().cpu().numpy()}
    if hc is not None:
        out["hc"] = hc.detach().double().cpu().numpy()
    for k in GRADS:
        if k == "V" and not dual:
            continue
        out["d" + k] = lv[k].grad.double().cpu().numpy()
    return out


def _oracle(inp, dual=True, K_iter=20, rounded=None):
    """float64 oracle (device-path semantics, padded rows zero) on the same values."""
    q = {k: inp[k] for k in inp}
    if rounded is not None:
        for k in ("Q", "K", "V"):
            q[k] = q[k].to(rounded)
    q = {k: (v.double() if isinstance(v, torch.Tensor) else v) for k, v in q.items()}
    g = tt.transport_grads(tt.transport_device, q["Q"], q["K"], q["x"], q["eps"], q["alpha"], q["r_h"],
                           V=q["V"] if dual else None, gxc=q["gxc"], ghc=q["ghc"] if dual else None,
                           K_iter=K_iter, mask=q.get("mask"), zero_pad_rows=True)
    names = dict(dQ="dQ", dK="dK", dx="dx", dalpha="dalpha", dr="dr_h", dV="dV", xc="xc", hc="hc")
    return {names[k]: v.numpy() for k, v in g.items()}


def _inputs(B, H, N, d, dv=None, seed=0, lengths=None, r_h=None):
    g = torch.Generator().manual_seed(seed)
    dv = dv or d
    inp = dict(Q=F.normalize(torch.randn(B, H, N, d, generator=g), dim=-1),
               K=F.normalize(torch.randn(B, H, N, d, generator=g), dim=-1),
               x=torch.randn(B, N, 3, generator=g) * 4.0, V=torch.randn(B, H, N, dv, generator=g),
               eps=torch.tensor([0.5, 1.0, 2.0, 4.0] * (H // 4) + [1.0] * (H % 4)),
               alpha=torch.randn(H, generator=g), r_h=r_h if r_h is not None else torch.full((H,), 10.0),
               gxc=torch.randn(B, H, N, 3, generator=g), ghc=torch.randn(B, H, N, dv, generator=g))
    if lengths is not None:
        m = torch.zeros(B, N)
        for b, L in enumerate(lengths):
            m[b, :L] = 1.0
        inp["mask"] = m
    return inp


def _check(got, ref, tol_out=2e-3, tol_grad=5e-3):
    """outputs: max-abs error <= tol_out; gradients: relative error <= tol_grad"""
    errs = {k: (float(np.abs(got[k] - ref[k]).max()) if k in ("xc", "hc") else rel_err(got[k], ref[k]))
            for k in ref if k in got}
    bad = {k: e for k, e in errs.items() if e > (tol_out if k in ("xc", "hc") else tol_grad)}
    assert not bad, "errors (outputs max-abs, gradients relative) " + ", ".join(f"{k} {e:.2e}" for k, e in errs.items())


@pytest.mark.parametrize("dual", [True, False])
def test_reference_device_path_golden(dual):
    inp, out = _golden()
    got = _run(inp, dual=dual)
    pre = "dual_" if dual else "single_"
    valid = inp["mask"].numpy() > 0.5
    rows = lambda a: np.concatenate([a[b][:, valid[b]].ravel() for b in range(a.shape[0])])  # noqa: E731
    assert np.abs(rows(got["xc"]) - rows(out[pre + "xc"])).max() <= 2e-3
    if dual:
        assert np.abs(rows(got["hc"]) - rows(out[pre + "hc"])).max() <= 2e-3
    # padded rows: 0 here (the reference's device path leaves a softmax there;
    # its trunk block multiplies them by the mask)
    assert np.abs(got["xc"][1][:, ~valid[1]]).max() == 0.0
    # gradients: the golden upstream gradient is nonzero on padded rows, where
    # the reference's outputs depend on the inputs and these are constant 0, so
    # the gradients are compared with the oracle's padded-rows-zero version (the
    # oracle itself is pinned to these golden gradients by test_oracle_transport)
    ref = _oracle(inp, dual=dual)
    _check(got, ref)


def test_bf16_resident_matches_oracle():
    inp = _inputs(2, 8, 256, 32, lengths=[256, 181], seed=1)
    _check(_run(inp, dtype=torch.bfloat16), _oracle(inp, rounded=torch.bfloat16))


def test_bf16_streamed_matches_oracle():
    # N > 384: the streamed kernels, with the geometry term and per-head r_h
    inp = _inputs(1, 4, 512, 32, seed=2, lengths=[470], r_h=torch.tensor([10.0, 3.0, 1.0, 25.0]))
    _check(_run(inp, dtype=torch.bfloat16), _oracle(inp, rounded=torch.bfloat16))


def test_head_dims_differ_and_d64():
    # d_h = 16 with D_V = 24 (both zero-padded inside); d_h = 64 streamed-width heads
    inp = _inputs(1, 4, 96, 16, dv=24, seed=3)
    _check(_run(inp, dtype=torch.bfloat16), _oracle(inp, rounded=torch.bfloat16))
    inp = _inputs(1, 4, 128, 64, seed=4, lengths=[100])
    _check(_run(inp, dtype=torch.bfloat16), _oracle(inp, rounded=torch.bfloat16))


def test_r_clamp_and_sign():
    # r_h = -4 (|r| used, gradient negated) and 0.05 (below the 0.1 clamp: no gradient)
    inp = _inputs(1, 4, 64, 32, seed=5, r_h=torch.tensor([10.0, -4.0, 0.05, 2.0]))
    got = _run(inp, dtype=torch.bfloat16)
    ref = _oracle(inp, rounded=torch.bfloat16)
    _check(got, ref)
    assert got["dr_h"][2] == 0.0
    assert np.sign(got["dr_h"][1]) == np.sign(ref["dr_h"][1]) != 0


def test_dual_vs_single_and_cpu_tensors():
    # reference tests/test_dual_transport.py: the dual's x_centroid equals the
    # single transport's (1e-4); CPU tensors in give CPU tensors out
    inp = _inputs(1, 8, 64, 32, seed=6)
    dev = torch.device("cuda")
    args = [inp[k].to(dev) for k in ("Q", "K", "x")]
    rest = [inp[k].to(dev) for k in ("eps", "alpha", "r_h")]
    xs = balanced_sinkhorn_transport(*args, *rest, K_iter=20)
    xd, hd = balanced_sinkhorn_transport_dual(*args, inp["V"].to(dev), *rest, K_iter=20)
    assert (xs - xd).abs().max().item() < 1e-4
    assert xs.dtype == torch.float32 and hd.shape == inp["V"].shape
    xcpu, hcpu = balanced_sinkhorn_transport_dual(inp["Q"], inp["K"], inp["x"], inp["V"], inp["eps"],
                                                  inp["alpha"], inp["r_h"], K_iter=20)
    assert xcpu.device.type == "cpu" and (xcpu - xd.cpu()).abs().max().item() < 1e-6


def test_deterministic():
    inp = _inputs(2, 4, 200, 32, seed=7, lengths=[200, 150])
    a = _run(inp, dtype=torch.bfloat16)
    b = _run(inp, dtype=torch.bfloat16)
    for k in a:
        assert np.array_equal(a[k], b[k]), k
