"""(batch, head)-sharded flash Sinkhorn: independent problems spread over GPUs.

The padded variable-length configuration (B=8, H=16, padded N=1024, true lengths L_b in [64, 1024])
holds B*H independent optimal-transport problems whose cost grows like L_b^2.
``partition_problems`` balances that cost over the ranks: the (b, h) pairs are
ordered by decreasing length (the longest-processing-time rule) and each rank
takes a contiguous run of about total/world cost, so the imbalance is at most
one problem's cost.  No data-path collective is needed.  ``rank_blocks`` turns
a rank's run into at most three rectangles of the length-sorted batch, so a
rank issues at most three kernel sequences per call, whatever B and H are: the
streamed path's cost per call is dominated by its launch count at these sizes.
"""

from __future__ import annotations

import torch

__all__ = ["partition_problems", "rank_blocks", "bh_sharded_flash_sinkhorn"]


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


def rank_blocks(lengths, H: int, world: int, rank: int):
    """This rank's share of partition_problems as rectangles of the batch sorted
    by decreasing length: returns (order, blocks) with `order` the batch
    permutation and blocks (s0, s1, h0, h1) over sorted positions [s0, s1) and
    heads [h0, h1).  Whole batch elements merge into one block, so a rank has at
    most three blocks (a partial element at each end of its run)."""
    order = sorted(range(len(lengths)), key=lambda b: -int(lengths[b]))
    pos = {b: i for i, b in enumerate(order)}
    blocks = []
    for b, h0, h1 in partition_problems(lengths, H, world)[rank]:
        sp = pos[b]
        if (blocks and h0 == 0 and h1 == H and blocks[-1][1] == sp and blocks[-1][2] == 0
                and blocks[-1][3] == H):
            blocks[-1] = (blocks[-1][0], sp + 1, 0, H)
        else:
            blocks.append((sp, sp + 1, h0, h1))
    return order, blocks


_streams: dict = {}


def _stream_pool(device, n):
    key = (device.index, n)
    if key not in _streams:
        _streams[key] = [torch.cuda.Stream(device) for _ in range(n)]
    return _streams[key]


def bh_sharded_flash_sinkhorn(Q, K, V, eps, log_mu, log_nu, K_iter, lam, lengths, world: int = 1, rank: int = 0,
                              mask=None, cg_opts=None, n_streams: int = 3):
    """This rank's (batch, head) share of flash_sinkhorn on the full (B, H, N, d)
    inputs.  The batch is first put in decreasing-length order (one gather,
    differentiable), then each block of rank_blocks runs as one call on a pool
    of `n_streams` CUDA streams (independent problems; autograd replays each
    backward on its forward's stream).  Returns (order, results) with results
    [(s0, s1, h0, h1, O, log_u, log_v)], O of shape (s1-s0, h1-h0, N, d) over the
    sorted batch positions; gradients reach the full Q, K, V."""
    from deepfold.model.kernels.sinkhorn_kernel import flash_sinkhorn

    order, blocks = rank_blocks(lengths, Q.shape[1], world, rank)
    if not blocks:
        return order, []
    idx = torch.tensor(order, device=Q.device)
    Qs, Ks, Vs = (t.index_select(0, idx) for t in (Q, K, V))
    lmu, lnu = log_mu.index_select(0, idx), log_nu.index_select(0, idx)
    ms = None if mask is None else mask.index_select(0, idx)
    cur = torch.cuda.current_stream(Q.device)
    pool = _stream_pool(Q.device, n_streams) if len(blocks) > 1 else [cur]
    res = []
    for i, (s0, s1, h0, h1) in enumerate(blocks):
        s = pool[i % len(pool)]
        s.wait_stream(cur)
        with torch.cuda.stream(s):
            O, _, lu, lv = flash_sinkhorn(Qs[s0:s1, h0:h1], Ks[s0:s1, h0:h1], Vs[s0:s1, h0:h1], None, None, None,
                                          eps[h0:h1], None, lmu[s0:s1, h0:h1], lnu[s0:s1, h0:h1], K_iter=K_iter,
                                          lam=lam, mask=None if ms is None else ms[s0:s1], cg_opts=cg_opts)
        for t in (O, lu, lv):
            t.record_stream(cur)
        res.append((s0, s1, h0, h1, O, lu, lv))
    for s in pool:
        if s is not cur:
            cur.wait_stream(s)
    return order, res
