"""Pins oracle/transport_torch.py against golden vectors of the reference's own
balanced transport (tests/golden/balanced_*.npz, made by make_golden.py): its
device path (the Triton kernels of flash_sinkhorn_transport.py, forward and
unrolled backward, run by Triton's CPU interpreter) on a padded batch, and its
CPU path (_sinkhorn_cpu under autograd) through the public API.  CPU only."""

import os

import numpy as np
import pytest
import torch

from oracle import transport_torch as tt

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def _load(name):
    z = np.load(os.path.join(GOLDEN, f"{name}.npz"))
    inp = {k[3:]: torch.tensor(z[k]).double() for k in z.files if k.startswith("in_")}
    out = {k[4:]: z[k].astype(np.float64) for k in z.files if k.startswith("out_")}
    return inp, out


def _close(a, b, rtol, what):
    a = np.asarray(a, np.float64)
    err = np.abs(a - b).max() / max(np.abs(b).max(), 1e-30)
    assert err <= rtol, f"{what}: max error {err:.3e} of the largest entry > {rtol}"


def test_device_path_dual_and_single():
    inp, out = _load("balanced_device")
    args = (inp["Q"], inp["K"], inp["x"], inp["eps"], inp["alpha"], inp["r_h"])
    g = tt.transport_grads(tt.transport_device, *args, V=inp["V"], gxc=inp["gxc"], ghc=inp["ghc"],
                           K_iter=20, mask=inp["mask"])
    _close(g["xc"].numpy(), out["dual_xc"], 2e-5, "x_centroid")
    _close(g["hc"].numpy(), out["dual_hc"], 2e-5, "h_centroid")
    for k in ("Q", "K", "x", "V", "alpha", "r_h"):
        key = {"alpha": "dalpha", "r_h": "dr"}.get(k, "d" + k)
        _close(g[key].numpy(), out["dual_d" + k], 2e-4, "dual d" + k)
    g = tt.transport_grads(tt.transport_device, *args, gxc=inp["gxc"], K_iter=20, mask=inp["mask"])
    _close(g["xc"].numpy(), out["single_xc"], 2e-5, "single x_centroid")
    for k in ("Q", "K", "x", "alpha", "r_h"):
        key = {"alpha": "dalpha", "r_h": "dr"}.get(k, "d" + k)
        _close(g[key].numpy(), out["single_d" + k], 2e-4, "single d" + k)


def test_device_path_keeps_padded_rows():
    # the reference's device path writes the softmax over valid columns into
    # padded rows too; the op here writes zeros there (zero_pad_rows)
    inp, out = _load("balanced_device")
    xc = tt.transport_device(inp["Q"], inp["K"], inp["x"], inp["eps"], inp["alpha"], inp["r_h"], K_iter=20,
                             mask=inp["mask"], zero_pad_rows=True)
    pad = inp["mask"].numpy() < 0.5
    assert pad.any() and np.abs(out["dual_xc"][1][:, pad[1]]).max() > 0
    assert np.abs(xc.numpy()[1][:, pad[1]]).max() == 0
    _close(xc.numpy()[1][:, ~pad[1]], out["dual_xc"][1][:, ~pad[1]], 2e-5, "valid rows")


def test_cpu_path():
    inp, out = _load("balanced_cpu")
    args = (inp["Q"], inp["K"], inp["x"], inp["eps"], inp["alpha"], inp["r_h"])
    g = tt.transport_grads(tt.transport_cpu, *args, V=inp["V"], gxc=inp["gxc"], ghc=inp["ghc"], K_iter=20)
    _close(g["xc"].numpy(), out["xc"], 2e-5, "x_centroid")
    _close(g["hc"].numpy(), out["hc"], 2e-5, "h_centroid")
    for k in ("Q", "K", "x", "V", "alpha", "r_h"):
        key = {"alpha": "dalpha", "r_h": "dr"}.get(k, "d" + k)
        _close(g[key].numpy(), out["d" + k], 2e-4, "d" + k)
    # the clamp: r_h = 0.05 < 0.1 gets no gradient, r_h = -4 the negated one
    assert out["dr_h"][2] == 0.0 and g["dr"][2] == 0.0


@pytest.mark.parametrize("mode", ["device", "cpu"])
def test_paths_agree_without_padding(mode):
    # with no padded points the two reference paths compute the same transport,
    # up to the distance convention (sqrt(|dx|^2 + 1e-8) vs max(|dx|, 1e-8)):
    # it moves the diagonal's geometry term by 1e-4 / (r + 1e-4), about 1e-3 at
    # the clamp r = 0.1 that this fixture's third head sits on
    inp, out = _load("balanced_cpu")
    fn = tt.transport_device if mode == "device" else tt.transport_cpu
    tol = 5e-4 if mode == "device" else 2e-5
    xc, hc = fn(inp["Q"], inp["K"], inp["x"], inp["eps"], inp["alpha"], inp["r_h"], K_iter=20, V=inp["V"])
    _close(xc.numpy(), out["xc"], tol, "x_centroid")
    _close(hc.numpy(), out["hc"], tol, "h_centroid")
