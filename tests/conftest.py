"""pytest configuration: the ``gpu`` marker and import paths.

``deepfold-linear_b200`` plays the role of the reference's ``src`` directory:
with it on ``sys.path`` the drop-in modules import under the reference's own
names (``deepfold.model.kernels.flash_sinkhorn_attn`` ...).
"""

import os
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG_ROOT = os.path.join(ROOT, "deepfold-linear_b200")
for p in (ROOT, PKG_ROOT):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200, sm_100a)")


import pytest  # noqa: E402


@pytest.fixture(autouse=True)
def _clear_device_status(request):
    """Each GPU test starts with the device's sticky status word at 0 (a test
    that provokes a device error or a CG cap must not leak it into the next)."""
    if request.node.get_closest_marker("gpu") is not None:
        import torch

        if torch.cuda.is_available():
            from deepfold import _native as nat

            nat.ext().take_status(True)
    yield
