"""GPU parity of the single-corner SpectralConv3d (scx_spectral_conv3d_fwd) against the
reference's own spectral_conv3d outputs (fixtures from spectral_conv_combo/reference_pytorch.py
on test_3d_accuracy.py's cases) and the float64 numpy oracle on further shapes.  Tolerance:
test_3d_accuracy.py's 1e-4 (Frobenius relative error), also applied to max-abs / max|ref|."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import scx_data
from conftest import load_golden
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4


def _close(ref, got):
    fro, mx = oracle.rel_errors(ref, got)
    assert fro <= TOL and mx <= TOL, f"frobenius rel {fro:.3e}, max-abs rel {mx:.3e}"


@pytest.mark.parametrize("name", ["tiny_8", "small_16"])
def test_conv3d_matches_reference_fixture(name, cuda_device):
    import spectral_conv_ops

    g = load_golden(f"conv3d_{name}.npz")
    modes = tuple(int(v) for v in g["modes"])
    y = spectral_conv_ops.spectral_conv3d_supa(torch.from_numpy(g["x"]), torch.from_numpy(g["w"]), *modes)
    assert y.device.type == "cpu" and y.shape == g["y"].shape
    _close(g["y"], y.numpy())


@pytest.mark.parametrize("shape", [
    (1, 3, 5, 6, 10, 9, (3, 4, 5)),      # odd D and W, every kept index
    (2, 4, 6, 8, 12, 16, (5, 7, 9)),     # Nyquist bin kept (m3 = W/2 + 1)
    (1, 2, 2, 4, 4, 4, (4, 4, 3)),       # the whole spectrum
])
def test_conv3d_shapes_vs_oracle(shape, cuda_device):
    import spectral_conv_ops

    B, Cin, Cout, D, H, W, modes = shape
    x = scx_data.gaussian((B, Cin, D, H, W), 90)
    w = torch.complex(scx_data.gaussian((Cin, Cout) + modes, 91), scx_data.gaussian((Cin, Cout) + modes, 92))
    y = spectral_conv_ops.spectral_conv3d_supa(x.to(cuda_device), w.to(cuda_device), *modes, to_cpu=False)
    assert y.is_cuda
    _close(oracle.spectral_conv3d_np(x.numpy(), w.numpy(), *modes), y.cpu().numpy())


def test_conv3d_rejects_bad_modes(cuda_device):
    import spectral_conv_ops

    x = torch.randn(1, 2, 4, 4, 6)
    w = torch.zeros(2, 2, 2, 2, 5, dtype=torch.cfloat)  # m3 = 5 > W/2 + 1 = 4
    with pytest.raises(RuntimeError):
        spectral_conv_ops.spectral_conv3d_supa(x, w, 2, 2, 5)
    with pytest.raises(ValueError):
        spectral_conv_ops.spectral_conv3d_supa(torch.randn(2, 4, 4, 6), w, 2, 2, 4)


@pytest.mark.parametrize("name", ["official3d_8", "official3d_overlap"])
def test_official3d_matches_reference_fixture(name, cuda_device):
    """spectral_conv_ops.SpectralConv3d (four corners) with the baseline module's own weights
    against official_baseline.py's SpectralConv3d outputs: overlapping corners (later ones
    win) and the Nyquist bin included."""
    import spectral_conv_ops

    g = load_golden(f"conv3d_{name}.npz")
    modes = tuple(int(v) for v in g["modes"])
    layer = spectral_conv_ops.SpectralConv3d(int(g["Cin"]), int(g["Cout"]), *modes)
    with torch.no_grad():
        for i in range(1, 5):
            getattr(layer, f"weights{i}").copy_(torch.from_numpy(g[f"w{i}"]))
    layer = layer.to(cuda_device)
    y = layer(torch.from_numpy(g["x"]).to(cuda_device))
    assert y.is_cuda and tuple(y.shape) == g["y"].shape
    _close(g["y"], y.cpu().numpy())


def test_official3d_state_dict_matches_baseline_names():
    import spectral_conv_ops

    layer = spectral_conv_ops.SpectralConv3d(2, 3, 2, 2, 2)
    assert list(layer.state_dict()) == ["weights1", "weights2", "weights3", "weights4"]
