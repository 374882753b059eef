"""Position bins on the GPU (reference: src/deepfold/model/position_encoding.py:7-52).

* ``compute_bins`` (the drop-in) against the reference's own output
  (tests/golden/position_bins.npz), batched and unbatched, bit-exact;
* ``flash_sinkhorn_attn`` with ``pos_bins=(chain_id, global_idx, bond_matrix)``,
  where the kernels evaluate each pair's bin themselves, against the same call
  with the int32 table from ``compute_bins``: outputs, potentials and all
  gradients (dpos_weight included) bitwise equal, on the resident (N <= 384)
  and streamed (N > 384, d = 64) kernels.
"""

import os

import numpy as np
import pytest
import torch

from deepfold.model.kernels.flash_sinkhorn_attn import flash_sinkhorn_attn
from deepfold.model.position_encoding import compute_bins

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def test_compute_bins_matches_reference():
    z = np.load(os.path.join(GOLD, "position_bins.npz"))
    dev = torch.device("cuda")
    ch, gx, bd = (torch.tensor(z["in_" + k], device=dev) for k in ("chain_id", "global_idx", "bond"))
    out = compute_bins(ch, gx, bd)
    assert out.dtype == torch.int32 and np.array_equal(out.cpu().numpy(), z["out_bins"])
    assert np.array_equal(compute_bins(ch[0], gx[0], bd[0]).cpu().numpy(), z["out_bins_unbatched"])
    # CPU tensors in, CPU tensors out
    cpu = compute_bins(*(torch.tensor(z["in_" + k]) for k in ("chain_id", "global_idx", "bond")))
    assert cpu.device.type == "cpu" and np.array_equal(cpu.numpy(), z["out_bins"])


def _inputs(B, H, N, d, seed, dtype):
    g = torch.Generator().manual_seed(seed)
    dev = torch.device("cuda")
    t = lambda *s: torch.randn(*s, generator=g)  # noqa: E731
    chain = torch.sort(torch.randint(0, 3, (B, N), generator=g), dim=1).values
    gidx = torch.cumsum(torch.randint(1, 4, (B, N), generator=g), dim=1) - 40
    bond = torch.rand(B, N, N, generator=g) < 0.03
    bond = bond | bond.transpose(1, 2)
    lens = [N, N - N // 5][:B]
    mask = torch.zeros(B, N)
    for b, L in enumerate(lens):
        mask[b, :L] = 1
    lm = torch.where(mask > 0, -torch.log(mask.sum(-1, keepdim=True)), torch.full_like(mask, -1e9))
    lm = lm[:, None, :].expand(B, H, N).contiguous()
    inp = dict(Q=t(B, H, N, d).to(dtype), K=t(B, H, N, d).to(dtype), V=t(B, H, N, d).to(dtype),
               G=t(B, H, N, d), x=t(B, N, 3) * 3.0, pw=t(H, 68) * 0.3, w=torch.rand(H, generator=g) * 0.5,
               eps=torch.tensor([0.5, 1.0, 2.0, 4.0] * (H // 4)), lm=lm, mask=mask,
               dO=t(B, N, H * d), dxc=t(B, H, N, 3))
    inp = {k: v.to(dev) for k, v in inp.items()}
    return inp, (chain.to(dev), gidx.to(dev), bond.to(dev))


def _call(inp, bins):
    leaves = {k: inp[k].clone().requires_grad_(True) for k in ("Q", "K", "V", "G", "x", "pw", "w")}
    o, xc, lu, lv = flash_sinkhorn_attn(leaves["Q"], leaves["K"], leaves["V"], leaves["G"], leaves["x"],
                                        leaves["pw"], bins, inp["eps"], leaves["w"], inp["lm"], inp["lm"],
                                        K_iter=12, lam=float("inf"), r_0=10.0, mask=inp["mask"])
    ((o * inp["dO"]).sum() + (xc * inp["dxc"]).sum()).backward()
    torch.cuda.synchronize()
    out = dict(o=o, xc=xc, lu=lu, lv=lv)
    out.update({"d" + k: v.grad for k, v in leaves.items()})
    return {k: v.detach().cpu() for k, v in out.items()}


@pytest.mark.parametrize("shape", [(2, 4, 96, 32, torch.bfloat16), (1, 4, 700, 64, torch.bfloat16)],
                         ids=["resident", "streamed"])
def test_in_kernel_bins_equal_table(shape):
    B, H, N, d, dtype = shape
    inp, (chain, gidx, bond) = _inputs(B, H, N, d, seed=N, dtype=dtype)
    table = compute_bins(chain, gidx, bond)
    a = _call(inp, table)
    b = _call(inp, (chain, gidx, bond))
    for k in a:
        assert torch.equal(a[k], b[k]), k
    assert a["dpw"].abs().max() > 0
