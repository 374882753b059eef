"""(batch, head)-sharded flash Sinkhorn: independent problems spread over GPUs.

BASELINE config 3 (B=8, H=16, padded N=1024, true lengths L_b in [64, 1024])
holds B*H independent optimal-transport problems whose cost grows like L_b^2.
``partition_problems`` balances that cost over the ranks and keeps each rank's
heads of one batch element contiguous, so every chunk it hands out is a plain
view Q[b, h0:h1] of the full tensors: no copies, no data-path collective.  The
order is by decreasing length (the longest-processing-time rule), each rank
takes a contiguous run of (b, h) pairs of about total/world cost, so the
imbalance is at most one problem's cost.
"""

from __future__ import annotations

import torch

__all__ = ["partition_problems", "bh_sharded_flash_sinkhorn"]


def partition_problems(lengths, H: int, world: int):
    """Chunks (b, h0, h1) per rank for B = len(lengths) batch elements of H heads,
    problem cost length^2, balanced over `world` ranks.  Returns a list of
    `world` lists; every (b, h) appears exactly once."""
    order = sorted(range(len(lengths)), key=lambda b: -int(lengths[b]))
    cost = [int(lengths[b]) ** 2 for b in order for _ in range(H)]
    total = float(sum(cost))
    items = [(b, h) for b in order for h in range(H)]
    bounds, acc, k = [0], 0.0, 1
    for i, c in enumerate(cost):
        acc += c
        while k < world and acc >= total * k / world:
            bounds.append(i + 1)
            k += 1
    while len(bounds) < world:
        bounds.append(len(items))
    bounds.append(len(items))
    out = []
    for r in range(world):
        chunks = []
        for b, h in items[bounds[r]:bounds[r + 1]]:
            if chunks and chunks[-1][0] == b and chunks[-1][2] == h:
                chunks[-1] = (b, chunks[-1][1], h + 1)
            else:
                chunks.append((b, h, h + 1))
        out.append(chunks)
    return out


_streams: dict = {}


def _stream_pool(device, n):
    key = (device.index, n)
    if key not in _streams:
        _streams[key] = [torch.cuda.Stream(device) for _ in range(n)]
    return _streams[key]


def bh_sharded_flash_sinkhorn(chunks, Q, K, V, eps, log_mu, log_nu, K_iter, lam, mask=None, cg_opts=None,
                              n_streams: int = 4):
    """Run flash_sinkhorn on this rank's chunks (from partition_problems) of the
    full (B, H, N, d) inputs; returns [(b, h0, h1, O, log_u, log_v)] with O etc.
    of shape (1, h1-h0, N, ...).  Gradients flow to the full Q, K, V through the
    views.  The chunks are independent, so they run on a pool of `n_streams`
    CUDA streams (one chunk alone may not fill the GPU); autograd runs each
    chunk's backward on the stream of its forward, and the outputs are ordered
    after all of them on the current stream."""
    from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn

    cur = torch.cuda.current_stream(Q.device)
    pool = _stream_pool(Q.device, n_streams) if len(chunks) > 1 else [cur]
    res = []
    for i, (b, h0, h1) in enumerate(chunks):
        s = pool[i % len(pool)]
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            O, _, lu, lv = flash_sinkhorn(Q[b:b + 1, h0:h1], K[b:b + 1, h0:h1], V[b:b + 1, h0:h1], None, None,
                                          None, eps[h0:h1], None, log_mu[b:b + 1, h0:h1], log_nu[b:b + 1, h0:h1],
                                          K_iter=K_iter, lam=lam, mask=None if mask is None else mask[b:b + 1],
                                          cg_opts=cg_opts)
        for t in (O, lu, lv):
            t.record_stream(cur)
        res.append((b, h0, h1, O, lu, lv))
    for s in pool:
        if s is not cur:
            cur.wait_stream(s)
    return res
