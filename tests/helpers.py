"""Shared helpers for the parity tests: seeded inputs in the shapes of the
benchmark configurations and comparison against the CPU oracle."""

from __future__ import annotations

import numpy as np
import torch

from oracle import sinkhorn_oracle as orc


def make_inputs(B, H, N, d, *, seed=0, dtype=torch.bfloat16, eps=1.0, uniform=True, lengths=None,
                valid=None, device="cuda"):
    """Q, K, V ~ N(0,1) cast to `dtype`; marginals uniform or softmax(N(0,1)) over
    valid positions (padded entries -1e9); optional per-sample valid lengths, or
    an explicit (B, N) 0/1 mask `valid` of any pattern."""
    g = torch.Generator().manual_seed(seed)
    Q = torch.randn(B, H, N, d, generator=g).to(dtype)
    K = torch.randn(B, H, N, d, generator=g).to(dtype)
    V = torch.randn(B, H, N, d, generator=g).to(dtype)
    mask = None
    if lengths is not None:
        mask = torch.zeros(B, N)
        for b, L in enumerate(lengths):
            mask[b, :L] = 1.0
    if valid is not None:
        mask = valid.float().cpu()
    valid = torch.ones(B, N) if mask is None else mask
    if uniform:
        cnt = valid.sum(-1, keepdim=True)
        lmu = torch.where(valid > 0, -torch.log(cnt), torch.full_like(valid, -1e9))[:, None, :].expand(B, H, N)
        lmu = lmu.contiguous()
        lnu = lmu.clone()
    else:
        z = torch.randn(B, H, N, generator=g)
        z = torch.where(valid[:, None, :] > 0, z, torch.full_like(z, -1e30))
        lmu = torch.where(valid[:, None, :] > 0, torch.log_softmax(z, -1), torch.full_like(z, -1e9))
        z = torch.randn(B, H, N, generator=g)
        z = torch.where(valid[:, None, :] > 0, z, torch.full_like(z, -1e30))
        lnu = torch.where(valid[:, None, :] > 0, torch.log_softmax(z, -1), torch.full_like(z, -1e9))
    epst = torch.full((H,), float(eps)) if np.isscalar(eps) else torch.tensor(eps, dtype=torch.float32)
    dO = torch.randn(B, H, N, d, generator=g)
    out = dict(Q=Q, K=K, V=V, eps=epst, log_mu=lmu, log_nu=lnu, mask=mask, dO=dO)
    return {k: (None if v is None else v.to(device)) for k, v in out.items()}


def oracle_run(inp, K_iter, lam, with_grad=True, grad_mode="unrolled", **extra):
    """Oracle forward (+ gradient of sum(O * dO)) on the same (bf16-rounded) inputs."""
    c = lambda t: None if t is None else t.detach().float().cpu().numpy()  # noqa: E731
    B, H, N, d = inp["Q"].shape
    dO_flat = None
    if with_grad:
        dO_flat = c(inp["dO"]).transpose(0, 2, 1, 3).reshape(B, N, H * d)
    res, gr = orc.flash_sinkhorn_attn(
        c(inp["Q"]), c(inp["K"]), c(inp["V"]), None, c(extra.get("x_res")), c(extra.get("pos_weight")),
        c(extra.get("pos_bins")), c(inp["eps"]), c(extra.get("w_dist")), c(inp["log_mu"]),
        c(inp["log_nu"]), K_iter=K_iter, lam=lam, r_0=extra.get("r_0", 10.0), mask=c(inp["mask"]),
        with_grad=with_grad, dO_flat=dO_flat, dxc=c(extra.get("dxc")), grad_mode=grad_mode)
    return res, gr


def max_abs(a, b):
    return float(np.max(np.abs(np.asarray(a, np.float64) - np.asarray(b, np.float64))))


def rel_err(a, b):
    a = np.asarray(a, np.float64)
    b = np.asarray(b, np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-30))
