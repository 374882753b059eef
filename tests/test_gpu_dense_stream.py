"""Dense-cost entry points beyond the resident kernels' range (N > 384, or V head
dims above 32): sinkhorn_solve and compute_transport_output streamed from the
caller's cost in HBM, against the reference's torch computation restated in
oracle/sinkhorn_torch.py (float64)."""

import math

import pytest
import torch

from oracle import sinkhorn_torch as ort

from deepfold.model.sinkhorn import compute_transport_output, sinkhorn_solve

pytestmark = pytest.mark.gpu

DEV = torch.device("cuda")


def dense_case(B, H, N, d, seed, lengths=None):
    """Symmetric uniform cost (as the reference's dense tests build it), log-softmax
    marginals over the valid points (-1e9 on padding), per-head eps 0.5 / 1 / 2."""
    g = torch.Generator().manual_seed(seed)
    C = torch.rand(B, H, N, N, generator=g)
    C = C + C.transpose(-1, -2)
    mask = None
    if lengths is not None:
        mask = (torch.arange(N)[None, :] < torch.tensor(lengths)[:, None]).float()
    z = torch.randn(2, B, H, N, generator=g)
    if mask is not None:
        z = torch.where(mask[None, :, None, :] > 0, z, torch.full_like(z, -1e30))
    lm = torch.log_softmax(z, dim=-1)
    if mask is not None:
        lm = torch.where(mask[None, :, None, :] > 0, lm, torch.full_like(lm, -1e9))
    eps = torch.tensor([0.5, 1.0, 2.0, 1.0][:H])
    V = torch.randn(B, H, N, d, generator=g)
    G = torch.randn(B, H, N, d, generator=g)
    x = torch.randn(B, N, 3, generator=g) * 4
    return C, lm[0], lm[1], eps, V, G, x, mask


def oracle_solve(C, lmu, lnu, eps, lam, K, mask, threshold=None):
    d64 = lambda t: None if t is None else t.double()  # noqa: E731
    return ort.sinkhorn_solve(C.double(), lmu.double(), lnu.double(), eps.double(), lam=lam, K=K, mask=d64(mask),
                              threshold=threshold)


@pytest.mark.parametrize("N", [520, 515])          # 16-byte rows (vector loads) and ragged rows
@pytest.mark.parametrize("lam", [1.0, math.inf])
def test_dense_solve_beyond_resident_range(N, lam):
    C, lmu, lnu, eps, _, _, _, mask = dense_case(2, 3, N, 8, seed=N, lengths=[N, 401])
    lu, lv = sinkhorn_solve(C.to(DEV), lmu.to(DEV), lnu.to(DEV), eps.to(DEV), lam=lam, K=15, mask=mask.to(DEV))
    ru, rv = oracle_solve(C, lmu, lnu, eps, lam, 15, mask)
    assert (lu.cpu().double() - ru).abs().max().item() <= 2e-4
    assert (lv.cpu().double() - rv).abs().max().item() <= 2e-4
    # padded potentials are exactly zero
    assert torch.all(lu[1, :, 401:] == 0) and torch.all(lv[1, :, 401:] == 0)


def test_dense_solve_unbatched_cpu_tensors():
    """(H, N, N) CPU tensors in, CPU tensors out, as the reference's callers pass them."""
    C, lmu, lnu, eps, _, _, _, _ = dense_case(1, 2, 700, 8, seed=3)
    lu, lv = sinkhorn_solve(C[0], lmu[0], lnu[0], eps[:2], lam=1.0, K=10)
    assert lu.device.type == "cpu" and lu.shape == (2, 700)
    ru, rv = oracle_solve(C, lmu, lnu, eps[:2], 1.0, 10, None)
    assert (lu.double() - ru[0]).abs().max().item() <= 2e-4
    assert (lv.double() - rv[0]).abs().max().item() <= 2e-4


def test_dense_early_stop_per_problem():
    """threshold: every problem stops once its L-inf change of a check is below the
    threshold; the result agrees with the full run to the threshold's order."""
    C, lmu, lnu, eps, _, _, _, _ = dense_case(2, 3, 448, 8, seed=11)
    args = (C.to(DEV), lmu.to(DEV), lnu.to(DEV), eps.to(DEV))
    lu1, lv1 = sinkhorn_solve(*args, lam=1.0, K=300, threshold=1e-4, check_every=2)
    lu2, lv2 = sinkhorn_solve(*args, lam=1.0, K=300)
    assert (lu1 - lu2).abs().max().item() <= 1e-2
    assert (lv1 - lv2).abs().max().item() <= 1e-2
    ru, rv = oracle_solve(C, lmu, lnu, eps, 1.0, 300, None)
    assert (lu2.cpu().double() - ru).abs().max().item() <= 2e-4


@pytest.mark.parametrize("N,d", [(600, 48), (515, 100), (300, 64)])
def test_dense_transport_output(N, d):
    """O = sigmoid(G) T_norm V, T_norm and x_centroid for V head dims above 32 and
    N above the resident range, padded rows zeroed."""
    C, lmu, lnu, eps, V, G, x, mask = dense_case(2, 2, N, d, seed=d, lengths=[N, N - 77])
    lu, lv = oracle_solve(C, lmu, lnu, eps[:2], 1.0, 5, mask)
    o, T, xc = compute_transport_output(V.to(DEV), G.to(DEV), lu.float().to(DEV), lv.float().to(DEV), C.to(DEV),
                                        eps[:2].to(DEV), x_res=x.to(DEV), mask=mask.to(DEV))
    ro, rT, rxc, _ = ort.compute_transport_output(V.double(), G.double(), lu, lv, C.double(), eps[:2].double(),
                                                  x_res=x.double(), mask=mask.double())
    assert o.shape == (2, N, 2 * d) and T.shape == (2, 2, N, N) and xc.shape == (2, 2, N, 3)
    assert (T.cpu().double() - rT).abs().max().item() <= 1e-6
    assert (o.cpu().double() - ro).abs().max().item() <= 1e-4
    assert (xc.cpu().double() - rxc).abs().max().item() <= 1e-4
    assert torch.all(o[1, N - 77:] == 0) and torch.all(T[1, :, N - 77:] == 0)
