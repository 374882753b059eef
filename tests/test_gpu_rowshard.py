"""Row-sharded flash Sinkhorn (sinkhorn_rowshard): the phase API (dfs_stream_op)
driven on one GPU reproduces the single-call streamed path, and, with two or
more GPUs, a torchrun/NCCL run agrees with the single-GPU result on every rank."""

import os
import subprocess
import sys

import pytest
import torch

from helpers import make_inputs

from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn
from deepfold.model.kernels.sinkhorn_rowshard import row_sharded_flash_sinkhorn

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _run_both(inp, K_iter, lam, cg):
    outs = []
    for fn in (flash_sinkhorn, row_sharded_flash_sinkhorn):
        leaves = [inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V")]
        if fn is flash_sinkhorn:
            O, _, lu, lv = fn(*leaves, None, None, None, inp["eps"], None, inp["log_mu"], inp["log_nu"],
                              K_iter=K_iter, lam=lam, mask=inp["mask"], cg_opts=cg)
        else:
            O, _, lu, lv = fn(*leaves, inp["eps"], inp["log_mu"], inp["log_nu"], K_iter=K_iter, lam=lam,
                              mask=inp["mask"], cg_opts=cg)
        grads = torch.autograd.grad(O, leaves, grad_outputs=inp["dO"])
        outs.append([O, lu, lv] + [g.float() for g in grads])
    torch.cuda.synchronize()
    return outs


def test_phase_api_on_one_gpu_reproduces_streamed_path():
    inp = make_inputs(2, 2, 700, 64, seed=31, eps=0.5, uniform=False, lengths=[700, 290])
    ref, got = _run_both(inp, 25, 1.0, dict(rtol=1e-6, atol=0.0, max_iter=40))
    for a, b in zip(ref, got):
        assert float((a - b).detach().abs().max()) <= 1e-5


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("batch", [1, 2])
def test_two_gpu_row_sharded_matches_single_gpu(batch):
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr", "127.0.0.1", "--master-port", str(29531 + batch),
           os.path.join(ROOT, "tests", "rowshard_worker.py")]
    env = dict(os.environ, RS_N="1000", RS_B=str(batch), NCCL_NVLS_ENABLE="0")
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-2000:] + r.stderr[-2000:]


def test_bh_blocks_on_streams_match_full_batch():
    """The (batch, head) share of every rank of a 3-GPU partition, run here one
    after another (sorted batch, blocks on a stream pool), gives the outputs
    and gradients of one full-batch call.  The grids differ (a smaller batch
    gets more column splits per row block), so each row's sums are added in
    another order: agreement to rounding, 1e-4 after 20 iterations at eps 0.5
    for outputs and potentials, 2e-3 of their scale for the bf16 gradients."""
    from deepfold.model.kernels.sinkhorn_bhshard import bh_sharded_flash_sinkhorn

    lengths = [600, 200, 520]
    inp = make_inputs(3, 4, 600, 64, seed=41, eps=0.5, uniform=False, lengths=lengths)
    cg = dict(rtol=1e-6, atol=0.0, max_iter=40)
    leaves = [inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V")]
    O, _, lu, lv = flash_sinkhorn(*leaves, None, None, None, inp["eps"], None, inp["log_mu"], inp["log_nu"],
                                  K_iter=20, lam=1.0, mask=inp["mask"], cg_opts=cg)
    ref_g = torch.autograd.grad(O, leaves, grad_outputs=inp["dO"])
    leaves2 = [inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V")]
    outs, gos = [], []
    for rank in range(3):
        order, res = bh_sharded_flash_sinkhorn(*leaves2, inp["eps"], inp["log_mu"], inp["log_nu"], 20, 1.0,
                                               lengths, 3, rank, mask=inp["mask"], cg_opts=cg)
        for s0, s1, h0, h1, Oc, luc, lvc in res:
            for k, sp in enumerate(range(s0, s1)):
                b = order[sp]
                assert float((Oc[k] - O[b, h0:h1]).detach().abs().max()) <= 1e-4
                assert float((luc[k] - lu[b, h0:h1]).abs().max()) <= 1e-4
                outs.append(Oc[k])
                gos.append(inp["dO"][b, h0:h1])
    got_g = torch.autograd.grad(outs, leaves2, grad_outputs=gos)
    torch.cuda.synchronize()
    for a, b in zip(ref_g, got_g):
        # the backward's accumulation products (dS K, dS^T Q, T^T dO) take their
        # tile operand as tf32, where a 1e-6 change of an element may flip its
        # rounding; the gradients then come back in the leaves' dtype (bf16)
        a, b = a.float(), b.float()
        assert float((a - b).abs().max()) <= 2e-3 * float(a.abs().max())
