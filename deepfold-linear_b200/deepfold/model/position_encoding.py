"""``compute_bins``: the 68-bin position / bond encoding on the GPU.

Drop-in for ``deepfold.model.position_encoding.compute_bins`` of the reference
(src/deepfold/model/position_encoding.py:7-52): same arguments, same (N, N) or
(B, N, N) int32 result,

    same chain, no bond:  clamp(global_idx_i - global_idx_j, -32, 32) + 32
    other chain, no bond: 65;  same chain, bond: 66;  other chain, bond: 67,

computed by the library (``dfs_compute_bins``).  The Sinkhorn operators can
skip the table altogether: pass ``pos_bins=(chain_id, global_idx,
bond_matrix)`` to ``flash_sinkhorn_attn`` / ``flash_sinkhorn`` and the kernels
evaluate each pair's bin where they use it.  CPU tensors are computed on the
current CUDA device and the result returned on the CPU (there is no CPU path).
"""

from __future__ import annotations

import torch

from deepfold import _native as nat

__all__ = ["compute_bins"]


def compute_bins(chain_id: torch.Tensor, global_idx: torch.Tensor, bond_matrix: torch.Tensor) -> torch.Tensor:
    """chain_id, global_idx (N,) or (B, N) int; bond_matrix (N, N) or (B, N, N)
    bool -> bins (N, N) or (B, N, N) int32 in [0, 67]."""
    unbatched = chain_id.dim() == 1
    if unbatched:
        chain_id, global_idx, bond_matrix = chain_id.unsqueeze(0), global_idx.unsqueeze(0), bond_matrix.unsqueeze(0)
    on_cpu = not chain_id.is_cuda
    if on_cpu:
        if not torch.cuda.is_available():
            raise RuntimeError("deepfold B200 ops run on a CUDA device; none is available (no CPU path)")
        dev = torch.device("cuda", torch.cuda.current_device())
        chain_id, global_idx, bond_matrix = chain_id.to(dev), global_idx.to(dev), bond_matrix.to(dev)
    bins = nat.ext().compute_bins(chain_id, global_idx, bond_matrix)
    if on_cpu:
        bins = bins.cpu()
    return bins.squeeze(0) if unbatched else bins
