"""Generate the golden vectors that pin ``oracle/sinkhorn_oracle.py``,
``oracle/sinkhorn_torch.py`` and ``oracle/transport_torch.py``.

Run from the repository root on a machine that has the reference source:

    python tests/golden/make_golden.py --ref <path to deepfold-linear>/src

Every output stored here is produced by the reference's own torch code
(``deepfold.model.sinkhorn.sinkhorn_solve`` / ``compute_transport_output``,
``deepfold.model.kernels.flash_sinkhorn_attn.flash_sinkhorn_attn`` on CPU, and
torch autograd through them, the gradient oracle the reference itself uses in
tests/test_triton_fallback_consistency.py:316-355; for the balanced transport,
``deepfold.model.kernels.flash_sinkhorn_transport``'s Triton kernels executed by
Triton's CPU interpreter, and its CPU path).  Inputs are drawn here from
seeded numpy generators and saved alongside, so the fixtures are
self-contained and the GPU box never needs the reference.
"""

from __future__ import annotations

import argparse
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))


def _t(a, torch, grad=False):
    t = torch.tensor(np.asarray(a), dtype=torch.float32)
    if grad:
        t.requires_grad_(True)
    return t


def dense_cost(torch, Q, K, x, pos_w, bins, w_dist, r_0):
    """C = -QK^T/sqrt(d) + pos_w[h, bins] + w_h d/(r_0+d), as the reference builds it
    for its dense gradient oracle (test_triton_fallback_consistency.py:327-335)."""
    B, H, N, d = Q.shape
    C = -(Q @ K.transpose(-1, -2)) / d ** 0.5
    if x is not None:
        diff = x[:, :, None, :] - x[:, None, :, :]
        dist = ((diff ** 2).sum(-1) + 1e-8).sqrt()
        C = C + w_dist[None, :, None, None] * (dist / (r_0 + dist))[:, None]
    if pos_w is not None:
        idx = bins.long()
        C = C + torch.stack([pos_w[:, idx[b]] for b in range(B)])
    return C


def run_dense(torch, ref, inp, K_iter, lam, r_0, use_gate, mask=None):
    """sinkhorn_solve + compute_transport_output with autograd (the survey's oracle)."""
    sinkhorn_solve = ref["sinkhorn_solve"]
    cto = ref["compute_transport_output"]
    Q = _t(inp["Q"], torch, True)
    K = _t(inp["K"], torch, True)
    V = _t(inp["V"], torch, True)
    G = _t(inp["G"], torch, True) if use_gate else torch.full(V.shape, 30.0)
    x = _t(inp["x"], torch, True) if "x" in inp else None
    pos_w = _t(inp["pos_w"], torch, True) if "pos_w" in inp else None
    bins = torch.tensor(inp["bins"]) if "bins" in inp else None
    w_dist = _t(inp["w_dist"], torch, True) if "w_dist" in inp else None
    eps = _t(inp["eps"], torch)
    lmu = _t(inp["log_mu"], torch)
    lnu = _t(inp["log_nu"], torch)
    mk = None if mask is None else _t(mask, torch)
    C = dense_cost(torch, Q, K, x, pos_w, bins, w_dist, r_0)
    lu, lv = sinkhorn_solve(C, lmu, lnu, eps, lam=lam, K=K_iter, mask=mk)
    o, _, xc = cto(V, G, lu, lv, C, eps, x_res=x, mask=mk)
    dO = _t(inp["dO"], torch)
    loss = (o * dO).sum()
    if x is not None and "dxc" in inp:
        loss = loss + (xc * _t(inp["dxc"], torch)).sum()
    loss.backward()
    out = dict(o=o.detach().numpy(), log_u=lu.detach().numpy(), log_v=lv.detach().numpy(),
               dQ=Q.grad.numpy(), dK=K.grad.numpy(), dV=V.grad.numpy())
    if xc is not None:
        out["xc"] = xc.detach().numpy()
    if use_gate:
        out["dG"] = G.grad.numpy()
    if x is not None:
        out["dx"] = x.grad.numpy()
    if pos_w is not None:
        out["dpos"] = pos_w.grad.numpy()
    if w_dist is not None:
        out["dw"] = w_dist.grad.numpy()
    return out


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=os.environ.get("DEEPFOLD_REF_SRC"),
                    help="the reference's src directory (or set DEEPFOLD_REF_SRC)")
    ap.add_argument("--balanced-only", action="store_true", help=argparse.SUPPRESS)
    args = ap.parse_args()
    if not args.ref:
        ap.error("pass --ref <reference src directory> or set DEEPFOLD_REF_SRC")
    sys.path.insert(0, args.ref)
    import torch  # noqa: E402
    from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve  # noqa: E402
    from deepfold.model.kernels.flash_sinkhorn_attn import flash_sinkhorn_attn  # noqa: E402

    torch.set_num_threads(4)
    ref = dict(sinkhorn_solve=sinkhorn_solve, compute_transport_output=compute_transport_output)

    def save(name, inp, out, **meta):
        path = os.path.join(HERE, f"{name}.npz")
        arrs = {f"in_{k}": np.asarray(v) for k, v in inp.items()}
        arrs.update({f"out_{k}": np.asarray(v) for k, v in out.items()})
        arrs.update({f"meta_{k}": np.asarray(v) for k, v in meta.items()})
        np.savez_compressed(path, **arrs)
        print(name, os.path.getsize(path), "bytes")

    if args.balanced_only:
        balanced_fixtures(torch, save)
        return

    # 1) pure QK^T cost, balanced, converged: dense path + autograd
    r = np.random.default_rng(101)
    B, H, N, d = 1, 2, 48, 16
    inp = dict(Q=r.standard_normal((B, H, N, d)), K=r.standard_normal((B, H, N, d)),
               V=r.standard_normal((B, H, N, d)), G=r.standard_normal((B, H, N, d)),
               eps=np.array([1.0, 0.5]), log_mu=np.full((B, H, N), -np.log(N)),
               log_nu=np.full((B, H, N), -np.log(N)), dO=r.standard_normal((B, N, H * d)))
    inp = {k: v.astype(np.float32) for k, v in inp.items()}
    save("pure_balanced", inp, run_dense(torch, ref, inp, 40, 1e6, 10.0, True),
         K_iter=40, lam=1e6, r_0=10.0)

    # 2) config 0 of the benchmark: B=1 H=4 N=128 d=32, eps=1, K=20, mu=nu=1/N, seed 0.
    #    Forward through the reference's flash_sinkhorn_attn (CPU path) with the
    #    position / geometry terms zeroed and the gate saturated; gradients from
    #    the dense path.
    g0 = torch.Generator().manual_seed(0)
    B, H, N, d = 1, 4, 128, 32
    Qt = torch.randn(B, H, N, d, generator=g0)
    Kt = torch.randn(B, H, N, d, generator=g0)
    Vt = torch.randn(B, H, N, d, generator=g0)
    inp = dict(Q=Qt.numpy(), K=Kt.numpy(), V=Vt.numpy(),
               eps=np.ones(H, np.float32), log_mu=np.full((B, H, N), -np.log(N), np.float32),
               log_nu=np.full((B, H, N), -np.log(N), np.float32),
               dO=torch.randn(B, N, H * d, generator=g0).numpy())
    gate = torch.full((B, H, N, d), 30.0)
    out = {}
    for lam, tag in ((1e6, "bal"), (1.0, "uot")):
        o, xc, lu, lv = flash_sinkhorn_attn(
            Qt, Kt, Vt, gate, torch.zeros(B, N, 3), torch.zeros(H, 68),
            torch.zeros(B, N, N, dtype=torch.int32), torch.tensor(inp["eps"]), torch.zeros(H),
            torch.tensor(inp["log_mu"]), torch.tensor(inp["log_nu"]), K_iter=20, lam=lam, r_0=10.0)
        dense = run_dense(torch, ref, inp, 20, lam, 10.0, False)
        out.update({f"o_{tag}": o.detach().numpy(), f"log_u_{tag}": lu.detach().numpy(),
                    f"log_v_{tag}": lv.detach().numpy(), f"dQ_{tag}": dense["dQ"],
                    f"dK_{tag}": dense["dK"], f"dV_{tag}": dense["dV"]})
    save("config0", inp, out, K_iter=20, r_0=10.0)

    # 3) full legacy-UOT feature set (position bins, geometry, gate, centroid,
    #    non-uniform marginals, per-head eps), lam = 1: reference flash_sinkhorn_attn
    #    forward (CPU path) + dense autograd gradients.
    r = np.random.default_rng(7)
    B, H, N, d = 2, 4, 24, 8
    inp = dict(Q=r.standard_normal((B, H, N, d)), K=r.standard_normal((B, H, N, d)),
               V=r.standard_normal((B, H, N, d)), G=r.standard_normal((B, H, N, d)),
               x=r.standard_normal((B, N, 3)) * 3.0, pos_w=r.standard_normal((H, 68)) * 0.3,
               eps=np.array([0.5, 1.0, 2.0, 4.0]), w_dist=r.random(H) * 0.5,
               log_mu=r.standard_normal((B, H, N)), log_nu=r.standard_normal((B, H, N)),
               dO=r.standard_normal((B, N, H * d)), dxc=r.standard_normal((B, H, N, 3)))
    inp = {k: v.astype(np.float32) for k, v in inp.items()}
    inp["log_mu"] = np.log(np.exp(inp["log_mu"]) / np.exp(inp["log_mu"]).sum(-1, keepdims=True)).astype(np.float32)
    inp["log_nu"] = np.log(np.exp(inp["log_nu"]) / np.exp(inp["log_nu"]).sum(-1, keepdims=True)).astype(np.float32)
    inp["bins"] = r.integers(0, 68, (B, N, N)).astype(np.int32)
    T = lambda k: torch.tensor(inp[k])  # noqa: E731
    o, xc, lu, lv = flash_sinkhorn_attn(T("Q"), T("K"), T("V"), T("G"), T("x"), T("pos_w"),
                                        T("bins"), T("eps"), T("w_dist"), T("log_mu"),
                                        T("log_nu"), K_iter=5, lam=1.0, r_0=10.0)
    out = dict(o=o.numpy(), xc=xc.numpy(), log_u=lu.numpy(), log_v=lv.numpy())
    dense = run_dense(torch, ref, inp, 5, 1.0, 10.0, True)
    for k in ("dQ", "dK", "dV", "dG", "dx", "dpos", "dw"):
        out[k] = dense[k]
    out["o_dense"] = dense["o"]
    save("uot_full", inp, out, K_iter=5, lam=1.0, r_0=10.0)

    # 4) padded variable-length batch with masks and non-uniform marginals
    #    (padded log-marginal -1e9 as tests/test_sinkhorn_batch.py:59-62).
    r = np.random.default_rng(3)
    B, H, N, d = 2, 2, 20, 8
    lens = [20, 13]
    mask = np.zeros((B, N), np.float32)
    lmu = np.full((B, H, N), -1e9)
    lnu = np.full((B, H, N), -1e9)
    for b, L in enumerate(lens):
        mask[b, :L] = 1
        for h in range(H):
            z = r.standard_normal(L)
            lmu[b, h, :L] = z - np.log(np.exp(z).sum())
            z = r.standard_normal(L)
            lnu[b, h, :L] = z - np.log(np.exp(z).sum())
    inp = dict(Q=r.standard_normal((B, H, N, d)), K=r.standard_normal((B, H, N, d)),
               V=r.standard_normal((B, H, N, d)), G=r.standard_normal((B, H, N, d)),
               eps=np.array([0.5, 1.0]), log_mu=lmu, log_nu=lnu,
               dO=r.standard_normal((B, N, H * d)), mask=mask)
    inp = {k: v.astype(np.float32) for k, v in inp.items()}
    save("masked_varlen", inp, run_dense(torch, ref, inp, 60, 1e6, 10.0, True, mask=inp["mask"]),
         K_iter=60, lam=1e6, r_0=10.0)

    # 5) dense-cost sinkhorn_solve with the L-inf early stop (sinkhorn.py:98-103)
    r = np.random.default_rng(11)
    B, H, N = 2, 2, 12
    C = np.abs(r.standard_normal((B, H, N, N))).astype(np.float32)
    lmu = np.log(r.dirichlet(np.ones(N), (B, H))).astype(np.float32)
    lnu = np.log(r.dirichlet(np.ones(N), (B, H))).astype(np.float32)
    eps = np.array([1.0, 2.0], np.float32)
    outs = {}
    for thr in (None, 1e-3):
        lu, lv = sinkhorn_solve(torch.tensor(C), torch.tensor(lmu), torch.tensor(lnu),
                                torch.tensor(eps), lam=1.0, K=100, threshold=thr, check_every=2)
        key = "none" if thr is None else "1e-3"
        outs["log_u_" + key] = lu.numpy()
        outs["log_v_" + key] = lv.numpy()
    save("solve_early_stop", dict(C=C, log_mu=lmu, log_nu=lnu, eps=eps), outs,
         K_iter=100, lam=1.0)

    # 7) position bins: the reference's compute_bins (position_encoding.py:7-52)
    #    on chains with gaps in the residue index, sparse bonds, batched and not
    from deepfold.model.position_encoding import compute_bins  # noqa: E402
    r = np.random.default_rng(31)
    B, N = 2, 57
    chain = np.sort(r.integers(0, 3, (B, N)), axis=1).astype(np.int64)
    gidx = np.cumsum(r.integers(1, 4, (B, N)), axis=1).astype(np.int64) - 30
    bond = r.random((B, N, N)) < 0.04
    bond = bond | bond.transpose(0, 2, 1)
    bins = compute_bins(torch.tensor(chain), torch.tensor(gidx), torch.tensor(bond))
    bins1 = compute_bins(torch.tensor(chain[0]), torch.tensor(gidx[0]), torch.tensor(bond[0]))
    save("position_bins", dict(chain_id=chain, global_idx=gidx, bond=bond),
         dict(bins=bins.numpy(), bins_unbatched=bins1.numpy()))

    env = dict(os.environ, TRITON_INTERPRET="1")
    subprocess.run([sys.executable, os.path.abspath(__file__), "--ref", args.ref, "--balanced-only"], env=env,
                   check=True)


def balanced_fixtures(torch, save):
    # 6) balanced transport of the trunk block (flash_sinkhorn_transport.py):
    #    the reference's device path -- its Triton kernels, forward and unrolled
    #    backward, run by Triton's CPU interpreter -- on a padded batch, and its
    #    CPU path (_sinkhorn_cpu under autograd) through the public API.  Triton
    #    reads the interpreter flag when its modules are imported, so this runs
    #    in a child process of its own (the flag would reroute the CPU paths of
    #    the fixtures above).
    from deepfold.model.kernels import flash_sinkhorn_transport as fst  # noqa: E402
    r = np.random.default_rng(23)
    B, H, N, d = 2, 4, 40, 16
    mask = np.ones((B, N), np.float32)
    mask[1, 27:] = 0
    unit = lambda a: a / np.linalg.norm(a, axis=-1, keepdims=True)  # noqa: E731
    inp = dict(Q=unit(r.standard_normal((B, H, N, d))), K=unit(r.standard_normal((B, H, N, d))),
               x=r.standard_normal((B, N, 3)) * 4.0, V=r.standard_normal((B, H, N, d)),
               eps=np.array([0.5, 1.0, 2.0, 4.0]), alpha=r.standard_normal(H),
               r_h=np.array([10.0, 3.0, 6.0, 0.5]), gxc=r.standard_normal((B, H, N, 3)),
               ghc=r.standard_normal((B, H, N, d)), mask=mask)
    inp = {k: v.astype(np.float32) for k, v in inp.items()}
    T = lambda k, g=False: _t(inp[k], torch, g)  # noqa: E731
    out = {}
    leaves = dict(Q=T("Q", True), K=T("K", True), x=T("x", True), V=T("V", True), alpha=T("alpha", True),
                  r_h=T("r_h", True))
    xc, hc = fst.BalancedSinkhornDualFn.apply(leaves["Q"], leaves["K"], leaves["x"], leaves["V"], T("eps"),
                                              leaves["alpha"], leaves["r_h"], 20, T("mask"))
    ((xc * T("gxc")).sum() + (hc * T("ghc")).sum()).backward()
    out.update(dual_xc=xc.detach().numpy(), dual_hc=hc.detach().numpy())
    out.update({f"dual_d{k}": v.grad.numpy() for k, v in leaves.items()})
    leaves = dict(Q=T("Q", True), K=T("K", True), x=T("x", True), alpha=T("alpha", True), r_h=T("r_h", True))
    xc = fst.BalancedSinkhornFn.apply(leaves["Q"], leaves["K"], leaves["x"], T("eps"), leaves["alpha"],
                                      leaves["r_h"], 20, T("mask"))
    (xc * T("gxc")).sum().backward()
    out["single_xc"] = xc.detach().numpy()
    out.update({f"single_d{k}": v.grad.numpy() for k, v in leaves.items()})
    save("balanced_device", inp, out, K_iter=20)

    #    CPU path through the public API, no mask; r_h with a negative entry and
    #    one below the 0.1 clamp
    inp2 = {k: v for k, v in inp.items() if k != "mask"}
    inp2["r_h"] = np.array([10.0, -4.0, 0.05, 2.0], np.float32)
    T = lambda k, g=False: _t(inp2[k], torch, g)  # noqa: E731
    leaves = dict(Q=T("Q", True), K=T("K", True), x=T("x", True), V=T("V", True), alpha=T("alpha", True),
                  r_h=T("r_h", True))
    xc, hc = fst.balanced_sinkhorn_transport_dual(leaves["Q"], leaves["K"], leaves["x"], leaves["V"], T("eps"),
                                                  leaves["alpha"], leaves["r_h"], K_iter=20)
    ((xc * T("gxc")).sum() + (hc * T("ghc")).sum()).backward()
    out = dict(xc=xc.detach().numpy(), hc=hc.detach().numpy())
    out.update({f"d{k}": v.grad.numpy() for k, v in leaves.items()})
    save("balanced_cpu", inp2, out, K_iter=20)



if __name__ == "__main__":
    main()
