"""``flash_sinkhorn``: the flash-Sinkhorn operator on the B200 C-ABI library.

Drop-in for ``deepfold.model.kernels.sinkhorn_kernel.flash_sinkhorn`` of the
reference (src/deepfold/model/kernels/sinkhorn_kernel.py:2385-2468): same
arguments, same batched/unbatched behaviour, same outputs
``(O_avg, x_centroid, log_u, log_v)``.

Differences from the reference, all deliberate:

* The backward is the implicit-function-theorem gradient solved by conjugate
  gradient on the device (``dfs_bwd``), not the K-step unrolled adjoint of
  sinkhorn_kernel.py:2086-2382.  At a converged forward both are equal.
* ``lam=float('inf')`` selects the balanced problem (kappa = 1 exactly); the
  reference computes lam/(lam+eps) and yields NaN there.
* Padded rows (mask 0) of ``x_centroid`` are 0, like the dense reference
  ``compute_transport_output`` (sinkhorn.py:175-177).
* Gradients with respect to ``log_u``/``log_v`` outputs are ignored, as in the
  reference backward (sinkhorn_kernel.py:2086).
* There is no CPU path.  CPU tensors (as the reference's own tests pass them)
  are computed on the current CUDA device and the results moved back to the
  CPU, differentiably; without a CUDA device the call raises.
* Head dims other than 32 and 64 (up to 64) run zero-padded inside the library.
* ``pos_bins`` may also be the tuple ``(chain_id, global_idx, bond_matrix)`` of
  ``compute_bins``' inputs (src/deepfold/model/position_encoding.py:7): the
  kernels then evaluate each pair's bin themselves and no (B, N, N) int32 table
  is built.
* Device-side errors (a bounded wait that gave up, non-finite potentials) are
  raised as RuntimeError by the first call that returns after the status has
  been read back (the status is read asynchronously), or at once by
  ``check_status()``; a CG solve that reached ``max_iter`` gives a warning.
"""

from __future__ import annotations

import math
import warnings

import torch

from deepfold import _native as nat

__all__ = ["flash_sinkhorn", "CG_DEFAULTS", "last_cg_report", "check_status"]

# CG stopping rule of the backward: ||r|| <= max(atol, rtol * ||r0||), as in
# deepfold.utils.cg.conjugate_gradient.
CG_DEFAULTS = dict(rtol=1e-6, atol=1e-10, max_iter=50)


def last_cg_report() -> dict:
    """Device tensors (cg_iters, cg_residual, status, fwd_status) of the most
    recent backward."""
    rep = nat.ext().last_report()
    if not rep:
        return {}
    cg, status, fwd_status = rep
    return dict(cg_iters=cg[0], cg_residual=cg[1].view(torch.float32), status=status, fwd_status=fwd_status)


def _raise_or_warn(bits: int) -> None:
    errs = bits & (nat.DFS_ERR_DEVICE_TIMEOUT | nat.DFS_ERR_NUMERIC)
    if bits & nat.DFS_WARN_CG_NOT_CONVERGED:
        warnings.warn("a previous flash_sinkhorn backward: CG reached max_iter for some problem; its gradient "
                      "is the last CG iterate", RuntimeWarning, stacklevel=3)
    if errs:
        raise RuntimeError(f"a previous flash_sinkhorn call reported a device error: {nat.status_string(errs)} "
                           f"(status {bits})")


def check_status(wait: bool = True) -> None:
    """Read the device status of the forward / backward calls made so far on the
    current device (all of them, once the current stream has drained, with
    ``wait``; otherwise those whose status has already been read back):
    RuntimeError for a device error, a RuntimeWarning for a CG solve that
    reached its iteration cap.  Calls raise for earlier device errors by
    themselves; this makes the check immediate."""
    _raise_or_warn(int(nat.ext().take_status(bool(wait))))


def _to_cuda(args: dict) -> dict:
    """CPU tensors of a call (also inside tuples) moved to the current CUDA device
    (autograd follows)."""
    if not torch.cuda.is_available():
        raise RuntimeError("deepfold B200 Sinkhorn ops run on a CUDA device; none is available (no CPU path)")
    dev = torch.device("cuda", torch.cuda.current_device())

    def mv(v):
        if isinstance(v, torch.Tensor):
            return v.to(dev)
        if isinstance(v, (tuple, list)):
            return tuple(mv(t) for t in v)
        return v
    return {k: mv(v) for k, v in args.items()}


def unsqueeze_bins(pos_bins):
    """pos_bins (a table or compute_bins' inputs) with a leading batch dim."""
    if pos_bins is None:
        return None
    if isinstance(pos_bins, (tuple, list)):
        return tuple(t.unsqueeze(0) for t in pos_bins)
    return pos_bins.unsqueeze(0)


def flash_sinkhorn(Q_ln, K_ln, V, x_res, pos_weight, pos_bins, eps, w_dist, log_mu, log_nu,
                   K_iter: int = 7, lam: float = 1.0, r_0: float = 10.0, log_u_init=None,
                   log_v_init=None, BLOCK_N: int = 64, mask=None, cg_opts: dict | None = None):
    """Flash-Sinkhorn forward (+ IFT/CG backward via autograd).

    Same signature as the reference (sinkhorn_kernel.py:2385); ``BLOCK_N`` is
    accepted and ignored (the kernels choose their own tiling).  ``x_res``,
    ``pos_weight``/``pos_bins`` and ``w_dist`` may be None to drop the
    centroid / position / geometry terms.  ``cg_opts`` overrides
    ``CG_DEFAULTS`` for the backward solve.

    Returns (O_avg (B,H,N,d) fp32, x_centroid (B,H,N,3) or None, log_u, log_v);
    unbatched (H,N,d) inputs give unbatched outputs.
    """
    del BLOCK_N
    if not Q_ln.is_cuda:
        a = _to_cuda(dict(Q_ln=Q_ln, K_ln=K_ln, V=V, x_res=x_res, pos_weight=pos_weight, pos_bins=pos_bins,
                          eps=eps, w_dist=w_dist, log_mu=log_mu, log_nu=log_nu, log_u_init=log_u_init,
                          log_v_init=log_v_init, mask=mask))
        out = flash_sinkhorn(a["Q_ln"], a["K_ln"], a["V"], a["x_res"], a["pos_weight"], a["pos_bins"], a["eps"],
                             a["w_dist"], a["log_mu"], a["log_nu"], K_iter=K_iter, lam=lam, r_0=r_0,
                             log_u_init=a["log_u_init"], log_v_init=a["log_v_init"], mask=a["mask"],
                             cg_opts=cg_opts)
        return tuple(None if t is None else t.cpu() for t in out)
    unbatched = Q_ln.dim() == 3
    if unbatched:
        Q_ln, K_ln, V = Q_ln.unsqueeze(0), K_ln.unsqueeze(0), V.unsqueeze(0)
        x_res = None if x_res is None else x_res.unsqueeze(0)
        pos_bins = unsqueeze_bins(pos_bins)
        log_mu, log_nu = log_mu.unsqueeze(0), log_nu.unsqueeze(0)
        log_u_init = None if log_u_init is None else log_u_init.unsqueeze(0)
        log_v_init = None if log_v_init is None else log_v_init.unsqueeze(0)
        mask = None if mask is None else mask.unsqueeze(0)
    if mask is not None:
        mask = mask.float()
    cg = dict(CG_DEFAULTS)
    if cg_opts:
        cg.update(cg_opts)
    if isinstance(lam, torch.Tensor):
        lam = float(lam)
    if not (lam > 0.0) or math.isnan(lam):
        raise ValueError("lam must be positive (inf for the balanced problem)")
    # native autograd function FlashSinkhornFn (csrc/dfs_torch.cpp): validates,
    # allocates and calls dfs_fwd / dfs_bwd of libdfsink on the current stream
    chain = gidx = bond = None
    if isinstance(pos_bins, (tuple, list)):
        chain, gidx, bond = pos_bins  # bins evaluated in the kernels
        pos_bins = None
    ext = nat.ext()
    out = ext.flash_sinkhorn(Q_ln, K_ln, V, x_res, pos_weight, pos_bins, eps, w_dist, log_mu,
                             log_nu, log_u_init, log_v_init, mask, int(K_iter), float(lam),
                             float(r_0), float(cg["rtol"]), float(cg["atol"]), int(cg["max_iter"]),
                             chain, gidx, bond)
    out = tuple(out) if len(out) == 4 else (out[0], None, out[1], out[2])
    _raise_or_warn(int(ext.take_status(False)))  # warnings found by the call's own check
    if unbatched:
        return tuple(None if t is None else t.squeeze(0) for t in out)
    return out
