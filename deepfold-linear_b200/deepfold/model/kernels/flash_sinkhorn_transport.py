"""Balanced Sinkhorn transport of the trunk block on the B200 library.

Drop-in for ``deepfold.model.kernels.flash_sinkhorn_transport`` of the
reference (src/deepfold/model/kernels/flash_sinkhorn_transport.py:376-545):
``balanced_sinkhorn_transport`` returns the transport-weighted coordinate
centroid, ``balanced_sinkhorn_transport_dual`` also the transport-weighted
features, with the reference's arguments and output shapes.

Per (batch, head) problem the cost is the cosine / geometry mix

    C_ij = (1 - w_h)(1 - q_i.k_j) + w_h dist_ij / (r_h + dist_ij),
    w_h = sigmoid(alpha_h),  r_h = max(|r_h param|, 0.1),
    dist_ij = sqrt(|x_i - x_j|^2 + 1e-8)

(flash_sinkhorn_transport.py:27-54), the iteration is balanced Sinkhorn with
uniform marginals, K_iter x (column update, row update) (``:298-310``), and the
outputs are x_centroid = T_norm x and h_centroid = T_norm V with T_norm the
row-normalised plan (``:117-169``, ``:171-243``).  Q_s and K_s are expected
L2-normalised along the head dim, as the trunk block passes them
(src/deepfold/model/trunk_block.py:170-177); nothing here depends on it.

The work runs in the native autograd function ``BalancedTransportFn``
(csrc/dfs_torch.cpp) on the same library calls as ``flash_sinkhorn``: the
constant part of the cost drops out of T_norm, the rest is the library's cost
at a per-head eps and geometry weight, the column-first order comes from
running the iteration on the transposed problem, and a second call writes the
outputs from those potentials.

Differences from the reference, all deliberate:

* The backward is the implicit-function-theorem gradient at the final
  potentials (device CG), not the K-step unrolled one
  (balanced_sinkhorn_bwd.py:36-404); both agree once the iteration has
  converged.  It returns gradients for Q_s, K_s, x_res, V_h, alpha_h and r_h
  (None for eps, K_iter, mask), like the reference.
* The gradient of r_h goes through max(|r_h|, 0.1) (sign, and 0 below 0.1), as
  the reference's CPU path (autograd) has it; its device kernels return the
  derivative with respect to the clamped value.
* Padded rows (mask 0) of both outputs are 0, as in the reference's CPU path
  (flash_sinkhorn_transport.py:271-279); its device path leaves them at the
  softmax over the valid columns.  The trunk block multiplies them by the mask.
* The marginals are 1/n per valid point of each batch element; the
  reference's device path uses one batch-mean constant (``:294``).  Constant
  marginals change only the column potential's offset, not T_norm.
* No CPU path: CPU tensors are computed on the current CUDA device and moved
  back, differentiably; without a CUDA device the call raises.
"""

from __future__ import annotations

import torch

from deepfold import _native as nat
from deepfold.model.kernels.sinkhorn_kernel import CG_DEFAULTS, _raise_or_warn, _to_cuda

__all__ = ["balanced_sinkhorn_transport", "balanced_sinkhorn_transport_dual"]


def _call(Q_s, K_s, x_res, V_h, eps, alpha_h, r_h, K_iter, mask, cg_opts):
    if not Q_s.is_cuda:
        a = _to_cuda(dict(Q_s=Q_s, K_s=K_s, x_res=x_res, V_h=V_h, eps=eps, alpha_h=alpha_h, r_h=r_h, mask=mask))
        out = _call(a["Q_s"], a["K_s"], a["x_res"], a["V_h"], a["eps"], a["alpha_h"], a["r_h"], K_iter, a["mask"],
                    cg_opts)
        return [t.cpu() for t in out]
    dev = Q_s.device
    eps, alpha_h, r_h = (torch.as_tensor(t, device=dev) for t in (eps, alpha_h, r_h))
    if mask is not None:
        mask = mask.to(dev)
    cg = dict(CG_DEFAULTS)
    if cg_opts:
        cg.update(cg_opts)
    ext = nat.ext()
    out = ext.balanced_transport(Q_s, K_s, x_res.to(dev), V_h, eps, alpha_h, r_h, mask, int(K_iter),
                                 float(cg["rtol"]), float(cg["atol"]), int(cg["max_iter"]))
    _raise_or_warn(int(ext.take_status(False)))
    return out


def balanced_sinkhorn_transport(Q_s: torch.Tensor, K_s: torch.Tensor, x_res: torch.Tensor,
                                eps: torch.Tensor, alpha_h: torch.Tensor, r_h: torch.Tensor,
                                K_iter: int = 20, mask: torch.Tensor | None = None,
                                cg_opts: dict | None = None) -> torch.Tensor:
    """Balanced Sinkhorn transport; returns x_centroid (B, H, N, 3).

    Q_s, K_s (B, H, N, d_h); x_res (B, N, 3); eps, alpha_h, r_h (H,);
    mask (B, N), 1 = real point (> 0.5 counts as real).  Same signature as the
    reference (flash_sinkhorn_transport.py:376); ``cg_opts`` overrides
    ``CG_DEFAULTS`` of the backward solve.  The output is fp32 (float64 for
    float64 inputs), as the reference's device path returns it.
    """
    return _call(Q_s, K_s, x_res, None, eps, alpha_h, r_h, K_iter, mask, cg_opts)[0]


def balanced_sinkhorn_transport_dual(Q_s: torch.Tensor, K_s: torch.Tensor, x_res: torch.Tensor,
                                     V_h: torch.Tensor, eps: torch.Tensor, alpha_h: torch.Tensor,
                                     r_h: torch.Tensor, K_iter: int = 20, mask: torch.Tensor | None = None,
                                     cg_opts: dict | None = None) -> tuple[torch.Tensor, torch.Tensor]:
    """Balanced Sinkhorn transport; returns (x_centroid (B, H, N, 3),
    h_centroid (B, H, N, D_V)) from one solve.

    V_h (B, H, N, D_V) with D_V <= 64; the other arguments as
    ``balanced_sinkhorn_transport`` (reference: flash_sinkhorn_transport.py:519).
    """
    xc, hc = _call(Q_s, K_s, x_res, V_h, eps, alpha_h, r_h, K_iter, mask, cg_opts)
    return xc, hc
