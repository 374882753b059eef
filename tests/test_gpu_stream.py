"""Parity of the streamed kernels (problems beyond the cluster-resident range:
N > 384 or d = 64, e.g. the var-len B=8 H=16 N=1024 and long N=8192 configurations) against the CPU oracle.

Same tolerances as the resident path: output max-abs <= 2e-3, marginal
residuals <= 1e-4 (the parity criterion).
"""

import numpy as np
import pytest
import torch

from helpers import make_inputs, max_abs, oracle_run
from test_gpu_forward import marginals, run

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-3
MARG_TOL = 1e-4


def check_forward(inp, K_iter, lam, pot_tol=2e-3, **kw):
    O, xc, lu, lv = run(inp, K_iter, lam, **kw)
    res, _ = oracle_run(inp, K_iter, lam, with_grad=False, **kw)
    assert max_abs(O.cpu().numpy(), res.O_avg) <= OUT_TOL
    assert max_abs(lu.cpu().numpy(), res.log_u) <= pot_tol
    assert max_abs(lv.cpu().numpy(), res.log_v) <= pot_tol
    return O, xc, lu, lv, res


def test_stream_d64_n1024_balanced():
    """Config 3 shapes without padding: N=1024, d=64, eps=0.5, balanced."""
    inp = make_inputs(1, 2, 1024, 64, seed=3, eps=0.5)
    _, _, lu, lv, _ = check_forward(inp, 30, float("inf"))
    assert marginals(inp, lu.cpu().numpy(), lv.cpu().numpy()) <= MARG_TOL


def test_stream_padded_varlen_unbalanced():
    """Config 3 style: padded variable lengths, non-uniform marginals, masks, kappa < 1."""
    inp = make_inputs(2, 2, 1024, 64, seed=4, eps=0.5, uniform=False, lengths=[1024, 333])
    O, _, lu, lv, _ = check_forward(inp, 30, 1.0)
    mask = inp["mask"].cpu().numpy()
    # padded rows and potentials are exact zeros
    assert np.all(O.cpu().numpy()[1, :, 333:] == 0.0)
    assert np.all(lu.cpu().numpy()[1, :, 333:] == 0.0) and np.all(lv.cpu().numpy()[1, :, 333:] == 0.0)
    assert mask[1, 333:].sum() == 0


def gapped_mask(N):
    """Batch 0: valid on [200, 260) and [300, 590) only (a leading gap longer than a
    tile, a hole, fully masked row blocks at both ends); batch 1: all valid."""
    m = torch.zeros(2, N)
    m[0, 200:260] = 1.0
    m[0, 300:590] = 1.0
    m[1] = 1.0
    return m


def test_stream_gapped_mask_skips_empty_tiles():
    """Tiles and row blocks outside a batch element's valid range are skipped;
    results still match the oracle, and masked rows are exact zeros."""
    inp = make_inputs(2, 2, 896, 64, seed=9, eps=0.5, uniform=False, valid=gapped_mask(896))
    O, _, lu, lv, _ = check_forward(inp, 25, 1.0)
    m = inp["mask"].cpu().numpy()[0] == 0
    assert np.all(O.cpu().numpy()[0][:, m] == 0.0)
    assert np.all(lu.cpu().numpy()[0][:, m] == 0.0) and np.all(lv.cpu().numpy()[0][:, m] == 0.0)


def test_stream_d32_ragged_tile():
    """d = 32 beyond the resident range, N not a multiple of the 128-column tile."""
    inp = make_inputs(1, 3, 700, 32, seed=5, eps=1.0)
    _, _, lu, lv, _ = check_forward(inp, 20, float("inf"))
    assert marginals(inp, lu.cpu().numpy(), lv.cpu().numpy()) <= MARG_TOL


def test_stream_centroid():
    inp = make_inputs(1, 2, 512, 64, seed=6, eps=1.0)
    g = torch.Generator().manual_seed(60)
    x = (torch.randn(1, 512, 3, generator=g) * 3.0).cuda()
    _, xc, _, _, res = check_forward(inp, 20, float("inf"), x_res=x)
    assert max_abs(xc.cpu().numpy(), res.xc) <= 5e-3


def test_stream_single_iteration_and_warm_start():
    """K = 1 from a warm start: exactly one row and one column half-update."""
    inp = make_inputs(1, 1, 640, 64, seed=8, eps=1.0)
    check_forward(inp, 1, float("inf"))


# ---------------------------------------------------------------- backward
from test_gpu_backward import check, grads  # noqa: E402
from helpers import rel_err  # noqa: E402


def test_stream_backward_d64_balanced():
    """Config 3 shapes, balanced: IFT/Schur-CG gradients vs the oracle's unrolled gradient."""
    inp = make_inputs(1, 2, 1024, 64, seed=11, eps=0.5)
    g = grads(inp, 60, float("inf"))
    _, ref = oracle_run(inp, 60, float("inf"))
    check(g, ref)


def test_stream_backward_padded_unbalanced_marginals():
    """Padded variable lengths, non-uniform marginals, kappa < 1, marginal gradients too."""
    inp = make_inputs(2, 2, 640, 64, seed=12, eps=0.5, uniform=False, lengths=[640, 301])
    g = grads(inp, 40, 1.0, want_marg=True)
    _, ref = oracle_run(inp, 40, 1.0)
    check(g, ref)
    for k in ("dlog_mu", "dlog_nu"):
        assert rel_err(g[k], ref[k]) <= 2e-2, k


def test_stream_backward_gapped_mask():
    """Backward with a gapped, non-prefix mask (empty tiles and row blocks skipped)."""
    inp = make_inputs(2, 2, 896, 64, seed=13, eps=0.5, uniform=False, valid=gapped_mask(896))
    g = grads(inp, 60, 1.0)
    _, ref = oracle_run(inp, 60, 1.0)
    check(g, ref)


def test_stream_backward_d32_ragged():
    inp = make_inputs(1, 2, 520, 32, seed=13, eps=1.0)
    g = grads(inp, 30, float("inf"))
    _, ref = oracle_run(inp, 30, float("inf"))
    check(g, ref)


def test_stream_backward_unconverged_matches_ift():
    """Few iterations: the kernel returns the fixed-point (IFT) gradient at those potentials."""
    inp = make_inputs(1, 1, 512, 64, seed=14, eps=1.0)
    g = grads(inp, 3, 1.0)
    _, ref = oracle_run(inp, 3, 1.0, grad_mode="ift")
    check(g, ref)
