"""Worker for tests/test_gpu_rowshard.py: run under torchrun with one rank per
GPU.  Every rank builds the same seeded inputs, runs the row-sharded forward +
backward over NCCL and the single-GPU path on its own GPU, and compares them.
Exit code 0 when all ranks agree within the forward / gradient tolerances."""

import math
import os
import sys
from datetime import timedelta

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, os.path.join(ROOT, "deepfold-linear_b200"))

import torch  # noqa: E402
import torch.distributed as dist  # noqa: E402

from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn  # noqa: E402
from deepfold.model.kernels.sinkhorn_rowshard import row_sharded_flash_sinkhorn  # noqa: E402


def main():
    local = int(os.environ["LOCAL_RANK"])
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=120), device_id=torch.device("cuda", local))
    rank = dist.get_rank()
    dev = torch.device("cuda", local)
    # B = 1 splits the forward's interleaved problem groups by head, B = 2 by batch element
    B, H, N, d = int(os.environ.get("RS_B", "1")), 4, int(os.environ.get("RS_N", "1000")), 64
    g = torch.Generator().manual_seed(5)
    Q, K, V = (torch.randn(B, H, N, d, generator=g).to(torch.bfloat16).to(dev) for _ in range(3))
    dO = torch.randn(B, H, N, d, generator=g).to(dev)
    mask = torch.ones(B, N)
    mask[0, N - 37:] = 0.0
    if B > 1:
        mask[1, N // 2:] = 0.0
    mask = mask.to(dev)
    lm = torch.where(mask > 0, -torch.log(mask.sum(-1, keepdim=True)), torch.full_like(mask, -1e9))
    lm = lm[:, None, :].expand(B, H, N).contiguous()
    eps = torch.full((H,), 0.5, device=dev)
    cg = dict(rtol=1e-6, atol=0.0, max_iter=40)
    outs = {}
    # single GPU, then the row-sharded run with each exchange of the half-updates'
    # potentials (peer memory, the default; NCCL all-gathers), twice each so that
    # a second call reuses the peer workspace and its counters
    for name in ("single", "peer", "peer", "collective"):
        os.environ["DFS_ROWSHARD_EXCHANGE"] = name
        leaves = [t.clone().requires_grad_(True) for t in (Q, K, V)]
        if name == "single":
            O, _, lu, lv = flash_sinkhorn(*leaves, None, None, None, eps, None, lm, lm, K_iter=30, lam=1.0,
                                          mask=mask, cg_opts=cg)
        else:
            O, _, lu, lv = row_sharded_flash_sinkhorn(*leaves, eps, lm, lm, K_iter=30, lam=1.0, mask=mask,
                                                      cg_opts=cg)
        grads = torch.autograd.grad(O, leaves, grad_outputs=dO)
        outs[name] = [O, lu, lv] + [t.float() for t in grads]
    torch.cuda.synchronize()
    bad = []
    for mode in ("peer", "collective"):
        for name, a, b, tol in zip(("O", "log_u", "log_v", "dQ", "dK", "dV"), outs["single"], outs[mode],
                                   (2e-3, 1e-3, 1e-3, 5e-3, 5e-3, 5e-3)):
            if name.startswith("d"):
                err = float((a - b).norm() / b.norm().clamp_min(1e-30))
            else:
                err = float((a - b).abs().max())
            if not (err <= tol):
                bad.append(f"{mode} {name} {err:.3e}")
    flag = torch.tensor([len(bad)], device=dev)
    dist.all_reduce(flag)
    print(f"rank {rank}: {'ok' if not bad else 'MISMATCH ' + ', '.join(bad)}", flush=True)
    dist.destroy_process_group()
    sys.exit(0 if int(flag.item()) == 0 else 1)


if __name__ == "__main__":
    main()
