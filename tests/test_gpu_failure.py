"""Failure detection on one GPU, in the forms that fault or hang nothing.

* A bounded device wait that runs out: a peer-exchange phase told to wait for
  more arrivals than any GPU will raise.  The waiting thread gives up after the
  library's 2 s bound, the kernel finishes its normal path, DFS_ERR_DEVICE_TIMEOUT
  is set in the status word, and the context stays usable.
* Non-finite input: a NaN in Q makes every column sum non-finite; the resident
  forward re-stabilises once, still fails, and reports DFS_ERR_NUMERIC, which the
  op raises as RuntimeError once the status has been read back: at once with
  check_status(), otherwise from the call that finds it (the next one, or the
  bad call itself if the read-back has already landed when it returns).
* A CG solve capped at one iteration reports DFS_WARN_CG_NOT_CONVERGED, which
  the op turns into a warning.
"""

import ctypes
import time

import pytest
import torch

from helpers import make_inputs

from deepfold import _native as nat
from deepfold.model.kernels.sinkhorn_kernel import check_status, flash_sinkhorn

pytestmark = pytest.mark.gpu


def _fwd_args(inp, lu, lv, O, status):
    return nat.DfsFwdArgs(Q=nat.ptr(inp["Q"]), K=nat.ptr(inp["K"]), V=nat.ptr(inp["V"]), eps=nat.ptr(inp["eps"]),
                          log_mu=nat.ptr(inp["log_mu"]), log_nu=nat.ptr(inp["log_nu"]), O=nat.ptr(O),
                          log_u=nat.ptr(lu), log_v=nat.ptr(lv), status=nat.ptr(status))


def test_peer_wait_that_runs_out_reports_timeout_and_returns():
    dev = torch.device("cuda")
    B, H, N, d = 1, 1, 128, 64
    inp = make_inputs(B, H, N, d, seed=3)
    prob = nat.make_problem(B, H, N, d, torch.bfloat16, 1, float("inf"), 10.0)
    fb, _ = nat.workspace_bytes(prob)
    ws = torch.zeros((fb + 255) // 4 + 64, device=dev, dtype=torch.float32)
    lu = torch.empty(B, H, N, device=dev)
    lv = torch.empty_like(lu)
    O = torch.empty(B, H, N, d, device=dev)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    args = _fwd_args(inp, lu, lv, O, status)
    peers = nat.DfsPeerSet(npeers=1, self=0, wait_for=0)
    peers.ws[0] = ws.data_ptr()
    lib = nat.lib()
    st = nat.stream_ptr(dev)
    # FWD_INIT raises this GPU's own arrival counter once
    nat.check(lib.dfs_stream_op_peer(nat.DFS_OP_FWD_INIT, prob, args, 0, N, ws.data_ptr(), fb, ctypes.byref(peers),
                                     st), "FWD_INIT")
    peers.wait_for = 1 + 1000  # arrivals that no GPU will ever raise
    torch.cuda.synchronize()
    t0 = time.monotonic()
    nat.check(lib.dfs_stream_op_peer(nat.DFS_OP_FWD_ROWS, prob, args, 0, N, ws.data_ptr(), fb, ctypes.byref(peers),
                                     st), "FWD_ROWS")
    torch.cuda.synchronize()
    took = time.monotonic() - t0
    assert int(status.item()) & nat.DFS_ERR_DEVICE_TIMEOUT
    assert 1.5 < took < 20.0, took
    # the context is intact: a regular call afterwards runs and reports nothing
    status.zero_()
    out = flash_sinkhorn(inp["Q"], inp["K"], inp["V"], None, None, None, inp["eps"], None, inp["log_mu"],
                         inp["log_nu"], K_iter=5, lam=float("inf"))
    torch.cuda.synchronize()
    assert torch.isfinite(out[0]).all()
    check_status()


def test_non_finite_input_raises():
    inp = make_inputs(1, 2, 96, 32, seed=4)
    Q = inp["Q"].clone()
    Q[0, 1, 7, 3] = float("nan")
    with pytest.raises(RuntimeError, match="non-finite"):
        flash_sinkhorn(Q, inp["K"], inp["V"], None, None, None, inp["eps"], None, inp["log_mu"], inp["log_nu"],
                       K_iter=5, lam=float("inf"))
        check_status()
    check_status()  # reported once: the status word starts again from 0


def test_non_finite_input_raises_on_the_next_call():
    inp = make_inputs(1, 2, 96, 32, seed=5)
    Q = inp["Q"].clone()
    Q[0, 0, 0, 0] = float("inf")
    with pytest.raises(RuntimeError, match="device error"):
        flash_sinkhorn(Q, inp["K"], inp["V"], None, None, None, inp["eps"], None, inp["log_mu"], inp["log_nu"],
                       K_iter=5, lam=float("inf"))
        torch.cuda.synchronize()  # the status read-back has landed
        flash_sinkhorn(inp["Q"], inp["K"], inp["V"], None, None, None, inp["eps"], None, inp["log_mu"],
                       inp["log_nu"], K_iter=5, lam=float("inf"))
    check_status()


@pytest.mark.parametrize("N,d", [(128, 32), (640, 64)])
def test_cg_iteration_cap_warns(N, d):
    inp = make_inputs(1, 2, N, d, seed=6, dtype=torch.float32)
    leaves = [inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V")]
    O, _, _, _ = flash_sinkhorn(*leaves, None, None, None, inp["eps"], None, inp["log_mu"], inp["log_nu"],
                                K_iter=20, lam=float("inf"), cg_opts=dict(max_iter=1, rtol=1e-12, atol=0.0))
    (O * inp["dO"]).sum().backward()
    with pytest.warns(RuntimeWarning, match="max_iter"):
        check_status()
    assert all(torch.isfinite(t.grad).all() for t in leaves)


def test_argument_errors_raise_cleanly():
    """Host-side rejections (head dim beyond 64; an invalid lam caught by the
    library's own validation) raise RuntimeError with the library's message."""
    from deepfold import _native as nat

    ext = nat.ext()
    dev = torch.device("cuda")
    lm = torch.zeros(1, 1, 64, device=dev)
    wide = torch.zeros(1, 1, 64, 96, device=dev)
    with pytest.raises(RuntimeError, match="outside the kernels' range"):
        ext.flash_sinkhorn(wide, wide, wide, None, None, None, torch.ones(1, device=dev), None, lm, lm, None, None,
                           None, 5, float("inf"), 10.0, 1e-6, 0.0, 50)
    x = torch.zeros(1, 1, 64, 32, device=dev)
    with pytest.raises(RuntimeError, match="invalid argument"):
        ext.flash_sinkhorn(x, x, x, None, None, None, torch.ones(1, device=dev), None, lm, lm, None, None, None, 5,
                           -1.0, 10.0, 1e-6, 0.0, 50)
    with pytest.raises(ValueError, match="lam"):
        flash_sinkhorn(x, x, x, None, None, None, torch.ones(1, device=dev), None, lm, lm, K_iter=5, lam=-1.0)
