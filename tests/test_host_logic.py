"""CPU: host-side logic of the drop-in API (no device calls)."""

from __future__ import annotations

import pytest
import torch

import scx_dist
import spectral_conv_ext
import spectral_conv_ops


@pytest.mark.parametrize("value,expected", [
    (True, True), (False, False), ("fused", True), ("sufft", True), ("supa", True), ("v1", False),
    ("cpu", False), (" Fused ", True),
])
def test_resolve_use_sufft_explicit(value, expected):
    assert spectral_conv_ops.resolve_use_sufft(64, 64, value) is expected


def test_resolve_use_sufft_auto_and_table():
    assert spectral_conv_ops.resolve_use_sufft(64, 128, "auto") is True
    assert spectral_conv_ops.resolve_use_sufft(32, 128, "auto") is False
    spectral_conv_ops._AUTO_TUNE_TABLE[32] = {"use_sufft": True}
    try:
        assert spectral_conv_ops.resolve_use_sufft(32, 128, "adaptive") is True
    finally:
        spectral_conv_ops._AUTO_TUNE_TABLE.clear()


def test_resolve_use_sufft_errors():
    with pytest.raises(ValueError):
        spectral_conv_ops.resolve_use_sufft(64, 64, "gpu")
    with pytest.raises(TypeError):
        spectral_conv_ops.resolve_use_sufft(64, 64, 1)


def test_input_rank_checked_before_device_use():
    w = torch.zeros(2, 2, 2, 2, dtype=torch.cfloat)
    with pytest.raises(ValueError):
        spectral_conv_ops.spectral_conv2d_supa(torch.zeros(2, 8, 8), w, w, 2, 2)


def test_ext_checks_raise_runtime_error():
    cpu = torch.zeros(1, 2, 2, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ext.spectral_mul(cpu, cpu)
    with pytest.raises(RuntimeError, match="last dim must be 2"):
        spectral_conv_ext.spectral_mul(torch.zeros(1, 2, 2, 2, 3), cpu)
    with pytest.raises(RuntimeError, match="float32"):
        spectral_conv_ext.spectral_mul(torch.zeros(1, 2, 2, 2, 2, dtype=torch.float64), cpu)
    with pytest.raises(RuntimeError, match="shape"):
        spectral_conv_ext.spectral_mul(torch.zeros(2, 2, 2, 2), cpu)


def test_module_parameters_match_reference_layout():
    torch.manual_seed(0)
    a = spectral_conv_ops.SpectralConv2dSupa(3, 4, 5, 6)
    torch.manual_seed(0)
    b = spectral_conv_ops.SpectralConv2d(3, 4, 5, 6)
    assert list(a.state_dict()) == ["weights1", "weights2"] == list(b.state_dict())
    assert a.weights1.shape == (3, 4, 5, 6) and a.weights1.dtype == torch.complex64
    assert torch.equal(a.weights1, b.weights1) and torch.equal(a.weights2, b.weights2)
    assert 0 <= a.weights1.real.min() and a.weights1.real.max() < 1.0 / 12
    assert 0 <= a.weights1.imag.min() and a.weights1.imag.max() < 1.0 / 12


@pytest.mark.parametrize("batch,world,expected", [
    (20, 8, [3, 3, 3, 3, 2, 2, 2, 2]), (16, 8, [2] * 8), (160, 8, [20] * 8), (3, 4, [1, 1, 1, 0]),
    (20, 1, [20]),
])
def test_shard_sizes(batch, world, expected):
    assert scx_dist.shard_sizes(batch, world) == expected
    ranges = [scx_dist.shard_range(batch, world, r) for r in range(world)]
    assert ranges[0][0] == 0 and ranges[-1][1] == batch
    assert all(ranges[i][1] == ranges[i + 1][0] for i in range(world - 1))


def test_fno_model_structure():
    import fno_model

    torch.manual_seed(0)
    m = fno_model.FNO2d(modes1=12, modes2=12, width=32, n_layers=4, in_channels=10)
    names = list(m.state_dict())
    assert names[:2] == ["lift.weight", "lift.bias"]
    assert "fourier_layers.3.spectral_conv.weights2" in names and names[-1] == "project.2.bias"
    with pytest.raises(ValueError):
        fno_model.FNO2d(n_layers=3)
    nn_free = fno_model.FNO2d(instance_norm=False)
    assert list(nn_free.state_dict()) == names


def test_official3d_module_construction_matches_baseline_fixture():
    """SpectralConv3d builds its four weight tensors in official_baseline.py's order: under the
    same torch.manual_seed they equal the weights the baseline module drew for the fixture."""
    import numpy as np
    import scx_data
    from conftest import load_golden

    for (name, B, Cin, Cout, D, H, W, modes, seed) in scx_data.OFFICIAL_3D_CASES:
        g = load_golden(f"conv3d_{name}.npz")
        torch.manual_seed(seed)
        layer = spectral_conv_ops.SpectralConv3d(Cin, Cout, *modes)
        assert list(layer.state_dict()) == ["weights1", "weights2", "weights3", "weights4"]
        for i in range(1, 5):
            assert np.array_equal(getattr(layer, f"weights{i}").detach().numpy(), g[f"w{i}"])
        x = torch.randn(B, Cin, D, H, W, generator=torch.Generator().manual_seed(seed + 1))
        assert np.array_equal(x.numpy(), g["x"])


def test_new_entry_points_check_arguments_before_device_use():
    w3 = torch.zeros(2, 2, 2, 2, 2, dtype=torch.cfloat)
    with pytest.raises(ValueError):
        spectral_conv_ops.spectral_conv3d_supa(torch.zeros(2, 4, 4, 6), w3, 2, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ext.spectral_conv3d_fwd(torch.zeros(1, 2, 4, 4, 6), w3, 2, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ext.spectral_conv2d_bwd(torch.zeros(1, 2, 8, 8), None, w3, w3, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ext.spectral_conv2d_fwd_saved(torch.zeros(1, 2, 8, 8), w3, w3, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ops.spectral_conv2d_autograd(torch.zeros(1, 2, 8, 8), w3, w3, 2, 2)
    with pytest.raises(RuntimeError, match="CUDA"):
        spectral_conv_ops.SpectralConv3d(2, 2, 2, 2, 2)(torch.zeros(1, 2, 4, 4, 6))
    with pytest.raises(RuntimeError, match="host tensor"):
        spectral_conv_ext.spectral_conv2d_fwd_host(torch.zeros(1, 2, 8, 8, dtype=torch.float64), w3, w3, 2, 2,
                                                   torch.device("cpu"))


def test_variant_table_round_trip(tmp_path):
    """scx_tune: a saved table reloads and is applied through the C ABI (no CUDA call);
    entries that do not apply to their shape are refused; merge replaces a shape's entry."""
    import _scx
    import scx_tune

    lib = _scx.lib
    lib.scx_clear_variants()
    assert lib.scx_dft_variants(128, 128, 16, 16) == (1 << 1) | (1 << 2) | (1 << 3)
    assert lib.scx_dft_variants(256, 256, 32, 32) == (1 << 1) | (1 << 3)
    assert lib.scx_dft_variants(96, 160, 16, 20) == 1 << 1
    assert lib.scx_dft_variants(64, 64, 65, 12) == 0  # m1 > H: invalid shape
    table = scx_tune.empty_table()
    scx_tune.merge(table, {"H": 64, "W": 64, "m1": 12, "m2": 12, "variant": "ffma"}, "dft")
    scx_tune.merge(table, {"H": 64, "W": 64, "m1": 12, "m2": 12, "variant": "tensor"}, "dft")  # replaces
    scx_tune.merge(table, {"H": 96, "W": 160, "m1": 16, "m2": 20, "variant": "tensor"}, "dft")  # not applicable
    scx_tune.merge(table, {"corners": 2, "B": 20, "Cin": 32, "Cout": 32, "modes": 256, "variant": 3}, "mix")
    assert len(table["dft"]) == 2
    path = scx_tune.save(table, tmp_path / "table.json")
    assert scx_tune.load(path) == 2
    assert lib.scx_get_variant(0, 64, 64, 12, 12, 0) == 2
    assert lib.scx_get_variant(0, 96, 160, 16, 20, 0) == 0
    assert lib.scx_get_variant(1, 2, 20, 32, 32, 256) == 3
    assert lib.scx_get_variant(1, 2, 20, 32, 32, 128) == -1
    assert lib.scx_set_mix_variant(2, 20, 32, 32, 256, 10) == 1  # out of range
    assert lib.scx_set_mix_variant(2, 20, 32, 32, 256, 9) == 0  # the tensor-core kernel
    assert lib.scx_get_variant(1, 2, 20, 32, 32, 256) == 9
    assert lib.scx_set_mix_variant(2, 20, 32, 32, 256, 3) == 0
    assert lib.scx_set_dft_variant(64, 64, 12, 12, 0) == 0 and lib.scx_get_variant(0, 64, 64, 12, 12, 0) == 0
    lib.scx_clear_variants()
    assert lib.scx_get_variant(1, 2, 20, 32, 32, 256) == -1
    assert scx_tune.load(tmp_path / "missing.json") == 0
