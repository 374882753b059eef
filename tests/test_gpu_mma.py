"""tcgen05 building block: D = A B^T with both operands K-major in 128B-swizzled
shared memory (tf32), issued by the same helper the kernels use, against torch
matmul in float64.  The shapes are those of the kernels' products."""

import pytest
import torch

from deepfold import _native as nat

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("N,K", [
    (192, 32),    # S = Q K^T, half of N=384 (two chained MMAs when N > 256)
    (384, 32),    # S over N=384 in one call
    (256, 64),
    (32, 384),    # O = T_norm V, dQ = dS K, dV = T_norm^T dO over N=384
    (64, 128),
])
def test_mma_kmajor(N, K):
    torch.manual_seed(1234 + N + K)
    dev = torch.device("cuda")
    A, B = torch.randn(64, K, device=dev), torch.randn(N, K, device=dev)
    ref = A.double() @ B.double().T
    D = torch.full((64, N), float("nan"), device=dev)
    nat.check(nat.lib().dfs_selftest_mma(0, A.data_ptr(), B.data_ptr(), D.data_ptr(), 64, N, K,
                                         nat.stream_ptr(dev)), "dfs_selftest_mma")
    torch.cuda.synchronize()
    assert torch.isfinite(D).all()
    err = (D.double() - ref).norm() / ref.norm()
    assert err < 2e-3, float(err)
