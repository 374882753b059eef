"""``flash_sinkhorn_attn``: gated flash-Sinkhorn attention on B200.

Drop-in for the reference entry point
``deepfold.model.kernels.flash_sinkhorn_attn.flash_sinkhorn_attn``
(src/deepfold/model/kernels/flash_sinkhorn_attn.py:670-795): it runs the
Sinkhorn transport (``flash_sinkhorn``, CUDA only) and applies the
``sigmoid(G)`` gate, the (B, N, H*d) permutation and the padding mask exactly as
the reference does (flash_sinkhorn_attn.py:776-795).  The reference's silent
CPU fallback (``FlashSinkhornAttn``, :751-774) does not exist here: CPU tensors
are computed on the current CUDA device (results come back on the CPU), and
without a CUDA device the call raises.
"""

from __future__ import annotations

import torch

from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn, unsqueeze_bins

__all__ = ["flash_sinkhorn_attn"]


def flash_sinkhorn_attn(Q_ln, K_ln, V, G, x_res, pos_weight, pos_bins, eps, w_dist, log_mu, log_nu,
                        K_iter: int = 7, lam: float = 1.0, r_0: float = 10.0, log_u_init=None,
                        log_v_init=None, mask=None, cg_opts: dict | None = None):
    """Gated Sinkhorn attention.

    Unbatched: Q_ln (H,N,d), x_res (N,3), pos_bins (N,N) ... -> o (N,H*d),
    x_centroid (H,N,3), log_u (H,N), log_v (H,N).  Batched: leading B.
    mask: (B,N) or (N,), 1 = real, 0 = padding.  pos_bins may also be the
    tuple (chain_id, global_idx, bond_matrix) of compute_bins' inputs.
    """
    unbatched = Q_ln.dim() == 3
    if unbatched:
        Q_ln, K_ln, V, G = Q_ln.unsqueeze(0), K_ln.unsqueeze(0), V.unsqueeze(0), G.unsqueeze(0)
        x_res = x_res.unsqueeze(0)
        pos_bins = unsqueeze_bins(pos_bins)
        log_mu, log_nu = log_mu.unsqueeze(0), log_nu.unsqueeze(0)
        log_u_init = None if log_u_init is None else log_u_init.unsqueeze(0)
        log_v_init = None if log_v_init is None else log_v_init.unsqueeze(0)
        mask = None if mask is None else mask.unsqueeze(0)
    B, H, N, d = Q_ln.shape
    if mask is None:
        mask = torch.ones(B, N, device=Q_ln.device, dtype=torch.float32)
    mask = mask.float()
    O_avg, x_centroid, log_u, log_v = flash_sinkhorn(
        Q_ln, K_ln, V, x_res, pos_weight, pos_bins, eps, w_dist, log_mu, log_nu, K_iter=K_iter,
        lam=lam, r_0=r_0, log_u_init=log_u_init, log_v_init=log_v_init, mask=mask, cg_opts=cg_opts)
    o_gated = torch.sigmoid(G.to(O_avg.device).float()) * O_avg
    mask = mask.to(O_avg.device)
    o_flat = o_gated.permute(0, 2, 1, 3).reshape(B, N, H * d) * mask.unsqueeze(-1)
    # padded duals are exactly 0 (the kernels write 0 there); the product keeps
    # the reference's own zeroing (flash_sinkhorn_attn.py:792-794)
    log_u = log_u * mask.unsqueeze(1)
    log_v = log_v * mask.unsqueeze(1)
    if unbatched:
        return (o_flat.squeeze(0), None if x_centroid is None else x_centroid.squeeze(0),
                log_u.squeeze(0), log_v.squeeze(0))
    return o_flat, x_centroid, log_u, log_v
