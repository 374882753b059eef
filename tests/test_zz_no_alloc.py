"""dfs_fwd_static: the forward for callers that cannot allocate device memory.

Such callers (a host program that only receives its buffers from another
runtime, an application whose device memory belongs to a framework's pool)
cannot hand the streamed kernels a workspace; dfs_fwd_static runs the same
forward on a fixed scratch array that the library keeps in device memory.
The test calls it through the C ABI twice in a row, on two different
problems, and checks each result against the regular dfs_fwd with a
caller-supplied workspace; it also checks that a problem needing more scratch
than the fixed array is refused before anything runs.  This file is collected
last, so a run that stops at the first failure has run every other test.
"""

import ctypes

import pytest
import torch

from deepfold import _native as nat

pytestmark = pytest.mark.gpu

OUT_TOL = 2e-3   # output max-abs tolerance of the forward parity tests
POT_TOL = 1e-3


def make_case(B, H, N, d, seed, lengths=None):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda", 0)
    t = {k: torch.randn(B, H, N, d, generator=g).to(torch.bfloat16).to(dev) for k in ("Q", "K", "V")}
    mask = None
    if lengths is not None:
        mask = torch.zeros(B, N)
        for b, L in enumerate(lengths):
            mask[b, :L] = 1.0
        mask = mask.to(dev)
    valid = torch.ones(B, N, device=dev) if mask is None else mask
    lm = torch.where(valid > 0, -torch.log(valid.sum(-1, keepdim=True)), torch.full_like(valid, -1e9))
    t["lm"] = lm[:, None, :].expand(B, H, N).contiguous()
    t["eps"] = torch.full((H,), 0.5, device=dev)
    t["mask"] = mask
    return t


def run(case, K_iter, lam, with_workspace):
    B, H, N, d = case["Q"].shape
    dev = case["Q"].device
    O = torch.full((B, H, N, d), float("nan"), device=dev)
    lu = torch.full((B, H, N), float("nan"), device=dev)
    lv = torch.full((B, H, N), float("nan"), device=dev)
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    prob = nat.make_problem(B, H, N, d, torch.bfloat16, K_iter, lam, 10.0)
    args = nat.DfsFwdArgs(Q=case["Q"].data_ptr(), K=case["K"].data_ptr(), V=case["V"].data_ptr(),
                          eps=case["eps"].data_ptr(), log_mu=case["lm"].data_ptr(), log_nu=case["lm"].data_ptr(),
                          mask=nat.ptr(case["mask"]), O=O.data_ptr(), log_u=lu.data_ptr(), log_v=lv.data_ptr(),
                          status=status.data_ptr())
    L = nat.lib()
    sp = torch.cuda.current_stream(dev).cuda_stream
    if with_workspace:
        fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
        nat.check(L.dfs_workspace_size(prob, ctypes.byref(fb), ctypes.byref(bb)), "dfs_workspace_size")
        ws = torch.empty(max(fb.value // 4, 1), device=dev, dtype=torch.float32)
        nat.check(L.dfs_fwd(prob, args, ws.data_ptr(), fb.value, sp), "dfs_fwd")
    else:
        nat.check(L.dfs_fwd_static(prob, args, sp), "dfs_fwd_static")
    torch.cuda.synchronize()
    assert int(status.item()) == 0
    return O, lu, lv


def compare(a, b):
    for x, y, tol in zip(a, b, (OUT_TOL, POT_TOL, POT_TOL)):
        assert torch.isfinite(x).all()
        assert float((x - y).abs().max()) <= tol


def test_static_scratch_forward_matches_dfs_fwd_on_two_calls():
    first = make_case(1, 2, 1024, 64, seed=21)                       # streamed, d = 64
    second = make_case(2, 2, 700, 32, seed=22, lengths=[700, 431])   # streamed, d = 32, padded
    for case, K_iter, lam in ((first, 20, float("inf")), (second, 15, 1.0)):
        ref = run(case, K_iter, lam, with_workspace=True)
        got = run(case, K_iter, lam, with_workspace=False)
        compare(got, ref)


def test_static_scratch_rejects_problems_beyond_its_size():
    big = nat.make_problem(8, 16, 16384, 64, torch.bfloat16, 10, 1.0, 10.0)  # needs about 1.7 GB
    fb, bb = ctypes.c_size_t(0), ctypes.c_size_t(0)
    L = nat.lib()
    assert L.dfs_workspace_size(big, ctypes.byref(fb), ctypes.byref(bb)) == nat.DFS_OK
    assert fb.value > nat.DFS_STATIC_SCRATCH_BYTES
    fake = nat.DfsFwdArgs(Q=16, K=16, V=16, eps=16, log_mu=16, log_nu=16, O=16, log_u=16, log_v=16)
    assert L.dfs_fwd_static(big, fake, None) == nat.DFS_ERR_WORKSPACE
