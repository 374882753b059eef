"""Dense-cost Sinkhorn surface: ``sinkhorn_solve`` and ``compute_transport_output``.

Drop-in for ``deepfold.model.sinkhorn`` of the reference
(src/deepfold/model/sinkhorn.py:17-198) on CUDA tensors.  The cost matrix C is
read by the same resident kernel as the flash path (``DFS_COST_DENSE``), so the
Sinkhorn loop never leaves the GPU:

* ``sinkhorn_solve``: log-domain (un)balanced iterations with the optional
  L-inf early stop.  The reference tests the stop condition once for the whole
  batch (one host sync per check); here every (batch, head) problem tests its
  own potentials on the device and stops independently, without a host sync.
  Problems that converge early therefore stop earlier than in the reference, a
  difference below ``threshold``.
* ``compute_transport_output``: row-normalised plan T_norm (materialised, as the
  reference returns it), gated output and optional centroid.

Problems of N <= 384 with V head dims up to 32 keep C on chip for the whole
loop (the cluster-resident kernel); all others -- N up to 65536, V head dims up
to 128 -- stream C from HBM once per half-iteration (csrc/dfs_dense.cu): the
cost is the input here, so those passes are bound by HBM bandwidth.

Both are differentiable, as the reference's are through autograd
(sinkhorn.py:30-36): with gradients wanted, ``sinkhorn_solve`` records every
iterate (csrc/dfs_dense_grad.cu, ``dfs_dense_iterate``) and its backward runs
the K-step adjoint as 2K passes over C (``dfs_dense_solve_bwd``) -- the exact
gradient of the iterations executed, as the reference's unrolled autograd.  With
``threshold`` set, that path stops where the reference stops: one batch-wide
test every ``check_every`` iterations (a host sync per test, as the reference
has).  ``compute_transport_output``'s backward forms dL/dT_norm with batched
products against V and x_res and runs the softmax backward of T_norm on the
device (``dfs_dense_transport_bwd``).  eps gets no gradient (a fixed per-head
constant in the reference); asking for one raises.  CPU tensors (as the
reference's tests pass them) are computed on the current CUDA device and the
results returned on the CPU; gradients flow back to the CPU leaves.
"""

from __future__ import annotations

import torch

from deepfold import _native as nat

__all__ = ["sinkhorn_solve", "compute_transport_output"]

DENSE_MAX_N = 1 << 16  # sequence length the dense-cost kernels accept
DENSE_MAX_D = 128      # head dim of V in compute_transport_output


def _on_gpu(fn):
    """Run ``fn`` on the current CUDA device when its cost tensor is on the CPU,
    returning CPU results (there is no CPU path)."""
    def wrapped(*args, **kw):
        first = args[0] if args else None
        if not isinstance(first, torch.Tensor) or first.is_cuda:
            return fn(*args, **kw)
        if not torch.cuda.is_available():
            raise RuntimeError("deepfold B200 Sinkhorn ops run on a CUDA device; none is available (no CPU path)")
        dev = torch.device("cuda", torch.cuda.current_device())
        mv = lambda t: t.to(dev) if isinstance(t, torch.Tensor) else t  # noqa: E731
        out = fn(*[mv(a) for a in args], **{k: mv(v) for k, v in kw.items()})
        return tuple(None if t is None else t.cpu() for t in out)
    wrapped.__doc__ = fn.__doc__
    wrapped.__name__ = fn.__name__
    return wrapped


def _dense_call(C, log_mu, log_nu, eps, lam, K, log_u_init, log_v_init, threshold, check_every,
                mask, V=None, x_res=None, want_T=False):
    dev = nat.require_cuda(C)
    B, H, N, _ = C.shape
    if N > DENSE_MAX_N:
        raise ValueError(f"N={N} exceeds the dense-cost kernels' range ({DENSE_MAX_N})")
    f32 = lambda t: None if t is None else t.detach().contiguous().float()  # noqa: E731
    # every tensor handed to the library is bound to a local name for the whole call
    Cc, lmu, lnu, epsc = f32(C), f32(log_mu), f32(log_nu), f32(eps)
    lui, lvi, mk, xr = f32(log_u_init), f32(log_v_init), f32(mask), f32(x_res)
    d = 32
    Vp = None
    if V is not None:
        d = V.shape[-1]
        if d > DENSE_MAX_D:
            raise ValueError(f"compute_transport_output supports head dims up to {DENSE_MAX_D}")
        Vp = f32(V)
    lu = torch.empty(B, H, N, device=dev, dtype=torch.float32)
    lv = torch.empty(B, H, N, device=dev, dtype=torch.float32)
    O = torch.empty(B, H, N, d, device=dev, dtype=torch.float32) if Vp is not None else None
    xc = torch.empty(B, H, N, 3, device=dev, dtype=torch.float32) if xr is not None else None
    T = torch.empty(B, H, N, N, device=dev, dtype=torch.float32) if want_T else None
    status = torch.zeros(1, device=dev, dtype=torch.int32)
    prob = nat.make_problem(B, H, N, d, torch.float32, K, lam, 10.0, cost_mode=nat.DFS_COST_DENSE,
                            threshold=threshold, check_every=check_every)
    args = nat.DfsFwdArgs(
        Q=None, K=None, V=nat.ptr(Vp), C=nat.ptr(Cc), x_res=nat.ptr(xr), pos_weight=None,
        pos_bins=None, eps=nat.ptr(epsc), w_dist=None, log_mu=nat.ptr(lmu), log_nu=nat.ptr(lnu),
        log_u_init=nat.ptr(lui), log_v_init=nat.ptr(lvi), mask=nat.ptr(mk), O=nat.ptr(O),
        x_centroid=nat.ptr(xc), log_u=nat.ptr(lu), log_v=nat.ptr(lv), status=nat.ptr(status),
        T_norm=nat.ptr(T))
    fwd_bytes, _ = nat.workspace_bytes(prob)  # copies of V when its head dim is transformed
    if N > 384 or d > 32:  # the HBM passes: room for the one-read iterations' column partials too
        fwd_bytes = (fwd_bytes + 255) // 256 * 256 + nat.lib().dfs_dense_work_bytes(B, H, N)
    ws = torch.empty((fwd_bytes + 3) // 4, device=dev, dtype=torch.float32) if fwd_bytes else None
    nat.check(nat.lib().dfs_fwd(prob, args, nat.ptr(ws), fwd_bytes, nat.stream_ptr(dev)), "dfs_fwd")
    return lu, lv, O, xc, T


def _wants_grad(*tensors) -> bool:
    return torch.is_grad_enabled() and any(isinstance(t, torch.Tensor) and t.requires_grad for t in tensors)


def _no_eps_grad(eps):
    if isinstance(eps, torch.Tensor) and eps.requires_grad and torch.is_grad_enabled():
        raise NotImplementedError("gradients with respect to eps are not provided (a fixed per-head constant)")


def _f32(t):
    return None if t is None else t.detach().float().contiguous()


def _chunk_ends(K: int, threshold, check_every: int) -> list[int]:
    """Iteration counts after which the differentiable forward returns to the
    host: K alone without a threshold; else every multiple of check_every (where
    the reference tests its stop condition, sinkhorn.py:98-103) and K."""
    if threshold is None:
        return [K]
    return sorted(set(range(check_every, K + 1, check_every)) | {K})


def _is_check(end: int, threshold, check_every: int) -> bool:
    """Whether the reference tests for convergence after iteration `end`."""
    return threshold is not None and end > 0 and end % check_every == 0


class _DenseSolveFn(torch.autograd.Function):
    """sinkhorn_solve with its unrolled adjoint (sinkhorn.py:82-110 under autograd)."""

    @staticmethod
    def forward(ctx, C, log_mu, log_nu, log_u_init, log_v_init, eps, mask, lam, K, threshold, check_every):
        dev = nat.require_cuda(C)
        B, H, N, _ = C.shape
        if N > DENSE_MAX_N:
            raise ValueError(f"N={N} exceeds the dense-cost kernels' range ({DENSE_MAX_N})")
        Cc, mu, nu, ep, mk = _f32(C), _f32(log_mu), _f32(log_nu), _f32(eps), _f32(mask)
        lui, lvi = _f32(log_u_init), _f32(log_v_init)
        n = B * H * N
        hist = torch.empty((2 * K + 2) * n, device=dev, dtype=torch.float32)
        lu = torch.empty(B, H, N, device=dev, dtype=torch.float32)
        lv = torch.empty_like(lu)
        status = torch.zeros(1, device=dev, dtype=torch.int32)
        change = torch.zeros(1, device=dev, dtype=torch.float32) if threshold is not None else None
        L, st = nat.lib(), nat.stream_ptr(dev)
        wbytes = L.dfs_dense_work_bytes(B, H, N)
        work = torch.empty((wbytes + 3) // 4, device=dev, dtype=torch.float32) if wbytes else None
        done, it = False, 0
        for end in _chunk_ends(K, threshold, check_every):
            nat.check(L.dfs_dense_iterate(B, H, N, float(lam), nat.ptr(Cc), nat.ptr(ep), nat.ptr(mu), nat.ptr(nu),
                                          nat.ptr(lui), nat.ptr(lvi), nat.ptr(mk), nat.ptr(hist), it, end,
                                          nat.ptr(lu), nat.ptr(lv), nat.ptr(change), nat.ptr(work),
                                          nat.ptr(status), st),
                      "dfs_dense_iterate")
            it = end
            if _is_check(end, threshold, check_every):
                done = float(change.item()) < threshold  # the reference's batch-wide test, one host sync
            if done:
                break
        ctx.iters, ctx.lam, ctx.shape = it, float(lam), (B, H, N)
        ctx.save_for_backward(Cc, mu, nu, ep, mk, hist)
        ctx.dtypes = [None if t is None else t.dtype for t in (C, log_mu, log_nu, log_u_init, log_v_init)]
        return lu, lv

    @staticmethod
    def backward(ctx, g_lu, g_lv):
        Cc, mu, nu, ep, mk, hist = ctx.saved_tensors
        B, H, N = ctx.shape
        dev = Cc.device
        need = ctx.needs_input_grad
        new = lambda shape, on: torch.empty(shape, device=dev, dtype=torch.float32) if on else None  # noqa: E731
        dC = new((B, H, N, N), need[0])
        dmu, dnu = new((B, H, N), need[1]), new((B, H, N), need[2])
        dlui, dlvi = new((B, H, N), need[3]), new((B, H, N), need[4])
        nbytes = nat.lib().dfs_dense_solve_bwd_scratch(B, H, N, ctx.iters)
        scratch = torch.empty((nbytes + 3) // 4, device=dev, dtype=torch.float32)
        gu, gv = _f32(g_lu), _f32(g_lv)
        nat.check(nat.lib().dfs_dense_solve_bwd(
            B, H, N, ctx.iters, ctx.lam, nat.ptr(Cc), nat.ptr(ep), nat.ptr(mu), nat.ptr(nu), nat.ptr(mk),
            nat.ptr(hist), nat.ptr(gu), nat.ptr(gv), nat.ptr(dC), nat.ptr(dmu), nat.ptr(dnu), nat.ptr(dlui),
            nat.ptr(dlvi), nat.ptr(scratch), nat.stream_ptr(dev)), "dfs_dense_solve_bwd")
        grads = [None if g is None else g.to(dt) for g, dt in zip((dC, dmu, dnu, dlui, dlvi), ctx.dtypes)]
        return (*grads, None, None, None, None, None, None)


class _DenseTransportFn(torch.autograd.Function):
    """T_norm, T_norm V and T_norm x_res of compute_transport_output (sinkhorn.py:152-194) with their backward."""

    @staticmethod
    def forward(ctx, V, log_u, log_v, C, eps, x_res, mask):
        B, H, N, d = V.shape
        zeros = torch.zeros(B, H, N, device=C.device, dtype=torch.float32)
        _, _, O, xc, T = _dense_call(C, zeros, zeros, _f32(eps), float("inf"), 0, _f32(log_u), _f32(log_v),
                                     None, 2, _f32(mask), V=V, x_res=x_res, want_T=True)
        ctx.save_for_backward(T, _f32(V), _f32(x_res), _f32(eps))
        ctx.dtypes = [t.dtype for t in (V, log_u, log_v, C)] + [None if x_res is None else x_res.dtype]
        return O, T, xc

    @staticmethod
    def backward(ctx, gO, gT, gxc):
        T, Vf, xr, ep = ctx.saved_tensors
        B, H, N, d = Vf.shape
        need = ctx.needs_input_grad
        dT = torch.matmul(gO.float(), Vf.transpose(-1, -2)) if gO is not None else torch.zeros_like(T)
        if gxc is not None and xr is not None:
            dT = dT + torch.matmul(gxc.float(), xr.transpose(-1, -2)[:, None])
        if gT is not None:
            dT = dT + gT.float()
        dT = dT.contiguous()
        dV = torch.matmul(T.transpose(-1, -2), gO.float()) if (need[0] and gO is not None) else None
        dx = None
        if need[5] and gxc is not None:
            dx = torch.matmul(T.transpose(-1, -2), gxc.float()).sum(1)
        dlv = torch.empty(B, H, N, device=T.device, dtype=torch.float32) if need[2] else None
        nat.check(nat.lib().dfs_dense_transport_bwd(B, H, N, nat.ptr(T), nat.ptr(dT), nat.ptr(ep), nat.ptr(dlv),
                                                    nat.stream_ptr(T.device)), "dfs_dense_transport_bwd")
        dlu = torch.zeros(B, H, N, device=T.device, dtype=ctx.dtypes[1]) if need[1] else None
        cast = lambda g, dt: None if g is None else g.to(dt)  # noqa: E731
        return (cast(dV, ctx.dtypes[0]), dlu, cast(dlv, ctx.dtypes[2]), cast(dT if need[3] else None, ctx.dtypes[3]),
                None, cast(dx, ctx.dtypes[4]), None)


@_on_gpu
def sinkhorn_solve(C, log_mu, log_nu, eps, lam: float = 1.0, K: int = 7, log_u_init=None,
                   log_v_init=None, threshold: float | None = None, check_every: int = 2, mask=None):
    """Log-domain Sinkhorn on a dense cost (H,N,N) or (B,H,N,N); returns (log_u, log_v)."""
    unb = C.dim() == 3
    if unb:
        C = C.unsqueeze(0)
        log_mu, log_nu = log_mu.unsqueeze(0), log_nu.unsqueeze(0)
        log_u_init = None if log_u_init is None else log_u_init.unsqueeze(0)
        log_v_init = None if log_v_init is None else log_v_init.unsqueeze(0)
        mask = None  # the reference ignores the mask for unbatched input
    f32 = lambda t: None if t is None else t.float().contiguous()  # noqa: E731
    if _wants_grad(C, log_mu, log_nu, log_u_init, log_v_init, eps):
        _no_eps_grad(eps)
        lu, lv = _DenseSolveFn.apply(C, log_mu, log_nu, log_u_init, log_v_init, eps, f32(mask), float(lam), int(K),
                                     threshold, int(check_every))
        if unb:
            return lu.squeeze(0), lv.squeeze(0)
        return lu, lv
    lu, lv, _, _, _ = _dense_call(C, f32(log_mu), f32(log_nu), f32(eps), float(lam), int(K),
                                  f32(log_u_init), f32(log_v_init), threshold, check_every, f32(mask))
    if unb:
        return lu.squeeze(0), lv.squeeze(0)
    return lu, lv


@_on_gpu
def compute_transport_output(V, G, log_u, log_v, C, eps, x_res=None, mask=None):
    """Gated transport output, T_norm and centroid (sinkhorn.py:115-198).

    Returns (o (B,N,H*d) or (N,H*d), T_norm, x_centroid or None).
    """
    unb = C.dim() == 3
    if unb:
        V, G, C = V.unsqueeze(0), G.unsqueeze(0), C.unsqueeze(0)
        log_u, log_v = log_u.unsqueeze(0), log_v.unsqueeze(0)
        x_res = None if x_res is None else x_res.unsqueeze(0)
        mask = None
    B, H, N, d = V.shape
    if _wants_grad(V, log_u, log_v, C, eps, x_res):
        _no_eps_grad(eps)
        if d > DENSE_MAX_D:
            raise ValueError(f"compute_transport_output supports head dims up to {DENSE_MAX_D}")
        O, T, xc = _DenseTransportFn.apply(V, log_u, log_v, C, eps, x_res, mask)
        o = torch.sigmoid(G.float()) * O
        o = o.permute(0, 2, 1, 3).reshape(B, N, H * d)
        if mask is not None:
            o = o * mask.float()[:, :, None]
        if unb:
            return o.squeeze(0), T.squeeze(0), None if xc is None else xc.squeeze(0)
        return o, T, xc
    zeros = torch.zeros(B, H, N, device=C.device, dtype=torch.float32)
    lu = log_u.float().contiguous()
    lv = log_v.float().contiguous()
    _, _, O, xc, T = _dense_call(C, zeros, zeros, eps.float().contiguous(), float("inf"), 0, lu, lv,
                                 None, 2, None if mask is None else mask.float().contiguous(),
                                 V=V, x_res=x_res, want_T=True)
    o = torch.sigmoid(G.float()) * O
    o = o.permute(0, 2, 1, 3).reshape(B, N, H * d)
    if mask is not None:
        o = o * mask.float()[:, :, None]
    if unb:
        return o.squeeze(0), T.squeeze(0), None if xc is None else xc.squeeze(0)
    return o, T, xc
