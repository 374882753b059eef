"""B200-native drop-in for the flash-Sinkhorn path of DeepFold-Linear.

Mirrors the reference package layout for that path only:

* ``deepfold.model.kernels.flash_sinkhorn_attn.flash_sinkhorn_attn``
* ``deepfold.model.kernels.sinkhorn_kernel.flash_sinkhorn``
* ``deepfold.model.sinkhorn.sinkhorn_solve``
* ``deepfold.utils.cg.conjugate_gradient`` / ``steihaug_cg``
* ``deepfold.sharding`` -- multi-GPU (batch, head) and row sharding

All Sinkhorn compute runs in ``libdfsink.so`` (hand-written sm_100a CUDA behind
the C ABI of ``include/dfsink.h``).
"""

__version__ = "0.1.0"
