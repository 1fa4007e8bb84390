"""CPU: pins the oracle restatements against fixtures produced by the reference itself
(tests/golden/make_golden.py ran spectral_conv/reference_pytorch.py and fno_ns/model.py)."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import scx_data
from conftest import GOLDEN, load_golden
from oracle import oracle

SPECTRAL_FIXTURES = sorted(p.name for p in GOLDEN.glob("spectral_*.npz"))
SMALL = {"spectral_refacc_tiny_8x8.npz", "spectral_refacc_small_32x32.npz", "spectral_refacc_target_64x64.npz",
         "spectral_spectral_b3_c24_100x72_m10.npz"}


def regenerate(g: dict):
    """Inputs of a fixture, rebuilt from its recipe (no reference code involved)."""
    B, Cin, Cout, H, W, m1, m2 = (int(g[k]) for k in ("B", "Cin", "Cout", "H", "W", "m1", "m2"))
    recipe = str(g["recipe"])
    if recipe == "reference_accuracy":
        x, w1, w2 = scx_data.reference_accuracy_case(B, Cin, Cout, H, W, m1, m2, int(g["seed"]))
    elif recipe == "reference_irregular":
        x, w1, w2, M = scx_data.reference_irregular_case(B, Cin, H, W)
        assert M == m1 == m2
    else:
        x, w1, w2, _ = scx_data.make_spectral_case(str(g["name"]))
    return x, w1, w2, (B, Cin, Cout, H, W, m1, m2)


def check_against_golden(g: dict, y: np.ndarray, tol: float) -> None:
    y = np.asarray(y, dtype=np.float64)
    if "y" in g:
        fro, mx = oracle.rel_errors(g["y"], y)
        assert fro <= tol and mx <= tol, (fro, mx)
    flat = y.reshape(-1)
    sv = g["sample_val"].astype(np.float64)
    assert np.abs(flat[g["sample_idx"]] - sv).max() <= tol * float(g["y_absmax"])
    norms = np.sqrt((y ** 2).sum(axis=(-2, -1)))
    assert np.abs(norms - g["y_plane_norm"]).max() <= tol * max(float(g["y_plane_norm"].max()), 1e-12)
    sums = y.sum(axis=(-2, -1))
    hw = y.shape[-1] * y.shape[-2]
    assert np.abs(sums - g["y_plane_sum"]).max() <= tol * float(g["y_absmax"]) * hw ** 0.5 + 1e-6


@pytest.mark.parametrize("fixture", SPECTRAL_FIXTURES)
def test_inputs_regenerate(fixture):
    g = load_golden(fixture)
    x, w1, w2, _ = regenerate(g)
    assert abs(x.double().sum().item() - float(g["x_sum"])) <= 1e-6 * max(1.0, abs(float(g["x_sum"])))
    assert abs(x.double().pow(2).sum().item() - float(g["x_sumsq"])) <= 1e-6 * float(g["x_sumsq"])
    assert abs(complex(w1.to(torch.complex128).sum().item()) - complex(g["w1_sum"])) <= 1e-9 * w1.numel()
    assert abs(complex(w2.to(torch.complex128).sum().item()) - complex(g["w2_sum"])) <= 1e-9 * w2.numel()
    if "x" in g:
        assert np.array_equal(x.numpy(), g["x"])


@pytest.mark.parametrize("fixture", SPECTRAL_FIXTURES)
def test_torch_port_matches_reference(fixture):
    g = load_golden(fixture)
    x, w1, w2, (B, Cin, Cout, H, W, m1, m2) = regenerate(g)
    y = oracle.spectral_conv2d_torch(x, w1, w2, m1, m2)
    check_against_golden(g, y.numpy(), 1e-5)


@pytest.mark.parametrize("fixture", sorted(SMALL))
def test_f64_direct_dft_matches_reference(fixture):
    g = load_golden(fixture)
    x, w1, w2, (B, Cin, Cout, H, W, m1, m2) = regenerate(g)
    y = oracle.spectral_conv2d_f64(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    # the reference computes in fp32: its own error (~3e-7) bounds the agreement
    check_against_golden(g, y, 1e-5)


def test_numpy_port_matches_reference():
    g = load_golden("spectral_spectral_b7_c20to36_96x160_m16x20.npz")
    x, w1, w2, (B, Cin, Cout, H, W, m1, m2) = regenerate(g)
    y = oracle.spectral_conv2d_np(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    check_against_golden(g, y, 1e-5)


@pytest.mark.parametrize("shape", [
    (2, 3, 4, 9, 11, 6, 6),    # 2*m1 > H: corner 2 overwrites corner 1, odd H and W
    (1, 2, 2, 7, 7, 7, 4),     # m1 = H, odd W with m2 = W//2+1
    (2, 3, 5, 12, 10, 4, 6),   # m2 = W//2+1 includes the Nyquist column (W even)
    (1, 1, 1, 1, 1, 1, 1),     # 1x1 grid
    (3, 5, 2, 16, 8, 1, 1),    # DC only
])
def test_f64_direct_dft_edge_cases(shape):
    B, Cin, Cout, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(B, Cin, H, W, generator=g)
    w1 = torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    ref = oracle.spectral_conv2d_np(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    got = oracle.spectral_conv2d_f64(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    np.testing.assert_allclose(got, ref, rtol=0, atol=1e-12 * max(1.0, np.abs(ref).max()))


def test_f64_corners_match_numpy_fft():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(2, 3, 10, 14, generator=g)
    c1, c2 = oracle.rfft2_corners_f64(x.numpy(), 4, 8)
    full = np.fft.rfft2(x.numpy().astype(np.float64))
    np.testing.assert_allclose(c1, full[:, :, :4, :8], atol=1e-10)
    np.testing.assert_allclose(c2, full[:, :, -4:, :8], atol=1e-10)


def test_oracle_rejects_bad_shapes():
    x = np.zeros((1, 1, 4, 4), dtype=np.float32)
    w = np.zeros((1, 1, 5, 2), dtype=np.complex64)
    with pytest.raises(ValueError):
        oracle.spectral_conv2d_f64(x, w, w, 5, 2)  # m1 > H
    w = np.zeros((1, 1, 2, 4), dtype=np.complex64)
    with pytest.raises(ValueError):
        oracle.spectral_conv2d_f64(x, w, w, 2, 4)  # m2 > W//2+1


def fno_state(seed: int):
    import fno_model

    fw = scx_data.FNO_WORKLOAD
    torch.manual_seed(seed)
    model = fno_model.FNO2d(modes1=fw["modes"], modes2=fw["modes"], width=fw["width"], n_layers=fw["layers"],
                            in_channels=fw["frames"])
    return model


def test_fno_init_and_oracle_match_reference():
    g = load_golden("fno_fno_ns_b20_w32_64x64_m12_l4.npz")
    model = fno_state(int(g["init_seed"]))
    sd = model.state_dict()
    assert list(sd.keys()) == [str(n) for n in g["param_names"]]
    for name, s in zip(g["param_names"], g["param_sums"]):
        v = sd[str(name)]
        got = complex(v.to(torch.complex128).sum().item()) if v.is_complex() else complex(v.double().sum().item())
        assert abs(got - complex(s)) <= 1e-9 * v.numel(), name
    fw = scx_data.FNO_WORKLOAD
    x_cl = scx_data.fno_input(fw["B"], fw["seed"], H=fw["H"], W=fw["W"], frames=fw["frames"])
    assert abs(x_cl.double().sum().item() - float(g["x_sum"])) <= 1e-6 * abs(float(g["x_sum"]))
    x = x_cl[..., : fw["frames"]].permute(0, 3, 1, 2).contiguous()
    y = oracle.fno2d_torch(sd, x, n_layers=fw["layers"], modes1=fw["modes"], modes2=fw["modes"])
    check_against_golden(g, y.detach().numpy(), 2e-5)
    # the module's own CPU path (the reference's use_supa=False path) agrees too
    with torch.no_grad():
        y2 = model(x, use_supa=False)
    check_against_golden(g, y2.numpy(), 2e-5)


@pytest.mark.parametrize("name", ["tiny_8", "small_16"])
def test_conv3d_oracle_matches_reference(name):
    """The numpy SpectralConv3d restatement against spectral_conv3d's own outputs
    (spectral_conv_combo/reference_pytorch.py:51-82) on test_3d_accuracy.py's cases, and the
    input recipe against the stored inputs."""
    g = load_golden(f"conv3d_{name}.npz")
    modes = tuple(int(v) for v in g["modes"])
    x, w = scx_data.reference_3d_case(int(g["B"]), int(g["Cin"]), int(g["Cout"]), int(g["D"]), int(g["H"]),
                                      int(g["W"]), modes, int(g["seed"]))
    assert np.array_equal(x.numpy(), g["x"]) and np.array_equal(w.numpy(), g["w"])
    y = oracle.spectral_conv3d_np(g["x"], g["w"], *modes)
    fro, mx = oracle.rel_errors(g["y"], y)
    assert fro <= 1e-5 and mx <= 1e-5, (fro, mx)


@pytest.mark.parametrize("name", ["official3d_8", "official3d_overlap"])
def test_official3d_oracle_matches_reference(name):
    """The numpy four-corner SpectralConv3d restatement against official_baseline.py's
    SpectralConv3d outputs, overlap and Nyquist cases included."""
    g = load_golden(f"conv3d_{name}.npz")
    modes = tuple(int(v) for v in g["modes"])
    y = oracle.spectral_conv3d_4c_np(g["x"], [g[f"w{i}"] for i in range(1, 5)], *modes)
    fro, mx = oracle.rel_errors(g["y"], y)
    assert fro <= 1e-5 and mx <= 1e-5, (fro, mx)
