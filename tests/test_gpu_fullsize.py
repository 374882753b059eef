"""Parity at the benchmark configurations' full size, through the bf16 path.

* B=8 H=16 padded N=1024 d=64, the bench's seeded variable lengths, softmax
  marginals over valid positions, eps=0.5, 50 iterations, balanced, CG tol
  1e-6 / max 50: the whole batch runs in one call with bf16 leaves; eight
  (batch, head) problems -- the shortest and the longest sample among them --
  are checked against the reference's own torch computation in float64
  (oracle/sinkhorn_torch.py: dense cost, sinkhorn_solve,
  compute_transport_output, autograd), outputs and potentials at 2e-3, dQ /
  dK / dV at 5e-3 relative, marginal residuals at 1e-4.
* B=1 H=16 N=8192 d=64, eps=1, 30 iterations, CG tol 1e-5 / max 40: the whole
  problem runs in one call; two heads are checked against the float64 checker
  with the implicit-function-theorem adjoint (autograd state at N=8192 would
  need ~30 GB of host memory per head; at this converged fixed point the
  implicit and the unrolled gradient agree to ~1e-6).

The bf16 leaves make the forward take the bf16 tensor-core path the model and
the bench use, and the gradients come back in bf16 as autograd returns them.
"""

import math

import numpy as np
import pytest
import torch

from bench import BIG, big_inputs
from helpers import max_abs, rel_err
from oracle import sinkhorn_torch as ort

from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn, last_cg_report

pytestmark = pytest.mark.gpu


def _run(c, host, mask, lmu, lnu):
    dev = torch.device("cuda")
    leaves = [host[k].to(dev).requires_grad_(True) for k in ("Q", "K", "V")]
    assert leaves[0].dtype == torch.bfloat16
    eps = torch.full((c["H"],), c["eps"], device=dev)
    O, _, lu, lv = flash_sinkhorn(*leaves, None, None, None, eps, None, lmu.to(dev), lnu.to(dev), K_iter=c["K_iter"],
                                  lam=c["lam"], mask=None if mask is None else mask.to(dev),
                                  cg_opts=dict(rtol=c["cg_rtol"], atol=0.0, max_iter=c["cg_max_iter"]))
    dQ, dK, dV = torch.autograd.grad(O, leaves, grad_outputs=host["dO"].to(dev).float())
    torch.cuda.synchronize()
    assert int(last_cg_report()["cg_iters"].max()) < c["cg_max_iter"]
    return [t.detach().float().cpu() for t in (O, lu, lv, dQ, dK, dV)]


@pytest.mark.timeout(900)
def test_config3_full_batch_bf16():
    c = BIG[3]
    host, lengths, mask, lmu, lnu = big_inputs(c)
    O, lu, lv, dQ, dK, dV = _run(c, host, mask, lmu, lnu)
    order = sorted(range(c["B"]), key=lambda b: lengths[b])
    picks = [(order[0], 0), (order[0], 15), (order[-1], 3), (order[-1], 12), (order[1], 7), (order[2], 9),
             (order[3], 1), (order[4], 14)]
    torch.set_num_threads(max(1, len(__import__("os").sched_getaffinity(0))))
    for b, h in picks:
        L = lengths[b]
        sl = (slice(b, b + 1), slice(h, h + 1))
        q, k, v = (host[n][sl].float().double() for n in ("Q", "K", "V"))
        dO = host["dO"][sl].float().double()
        eps = torch.tensor([c["eps"]], dtype=torch.float64)
        # the reference's arithmetic: lam = 1e6 (kappa = 1 - 1e-6; its formula is NaN at inf)
        O_r, lu_r, lv_r, dQ_r, dK_r, dV_r = ort.attn_fwd_bwd(q, k, v, eps, lmu[sl].double(), lnu[sl].double(),
                                                             c["K_iter"], 1e6, dO, dtype=torch.float64,
                                                             mask=mask[b:b + 1].double())
        what = f"(b={b}, h={h}, L={L})"
        assert max_abs(O[b, h], O_r[0, 0]) <= 2e-3, what
        assert max_abs(lu[b, h, :L], lu_r[0, 0, :L]) <= 2e-3, what
        assert max_abs(lv[b, h, :L], lv_r[0, 0, :L]) <= 2e-3, what
        assert np.all(lu[b, h, L:].numpy() == 0) and np.all(O[b, h, L:].numpy() == 0), what
        for got, ref, name in ((dQ, dQ_r, "dQ"), (dK, dK_r, "dK"), (dV, dV_r, "dV")):
            assert rel_err(got[b, h], ref[0, 0]) <= 5e-3, f"{name} {what}"
        r, cres = ort.marginal_residuals(q, k, eps, lu[sl], lv[sl], lmu[sl], lnu[sl], mask=mask[b:b + 1])
        assert r <= 1e-4 and cres <= 1e-4, f"marginals {what}: {r:.2e} {cres:.2e}"


@pytest.mark.timeout(900)
def test_config4_full_problem_bf16():
    c = BIG[4]
    host, _, _, lmu, lnu = big_inputs(c)
    O, lu, lv, dQ, dK, dV = _run(c, host, None, lmu, lnu)
    torch.set_num_threads(max(1, len(__import__("os").sched_getaffinity(0))))
    for h in (0, 11):
        q, k, v, dO = (host[n][0, h].float().double() for n in ("Q", "K", "V", "dO"))
        a = lmu[0, h].double()
        ref = ort.problem_fwd_bwd_ift(q, k, v, dO, c["eps"], a, lnu[0, h].double(), c["K_iter"], c["lam"])
        assert ref["marg_row"] <= 1e-6 and ref["marg_col"] <= 1e-6  # the checker's own fixed point
        assert max_abs(O[0, h], ref["O"]) <= 2e-3, h
        assert max_abs(lu[0, h], ref["log_u"]) <= 2e-3, h
        assert max_abs(lv[0, h], ref["log_v"]) <= 2e-3, h
        for got, name in ((dQ, "dQ"), (dK, "dK"), (dV, "dV")):
            assert rel_err(got[0, h], ref[name]) <= 5e-3, f"{name} h={h}"
        r, cres = ort.marginal_residuals(q[None, None], k[None, None], torch.tensor([c["eps"]], dtype=torch.float64),
                                         lu[0:1, h:h + 1], lv[0:1, h:h + 1], a[None, None], lnu[0:1, h:h + 1])
        assert r <= 1e-4 and cres <= 1e-4, f"marginals h={h}: {r:.2e} {cres:.2e}"
