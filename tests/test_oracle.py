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


def test_gradient_oracle_matches_finite_differences():
    """The backward's oracle (float64 autograd of the reference recipe) against central
    differences of the forward, on a small case with overlapping corners and odd W."""
    torch.manual_seed(0)
    B, Cin, Cout, H, W, m1, m2 = 1, 2, 3, 6, 7, 4, 3
    x = torch.randn(B, Cin, H, W, dtype=torch.float64)
    w1 = torch.randn(Cin, Cout, m1, m2, dtype=torch.complex128)
    w2 = torch.randn(Cin, Cout, m1, m2, dtype=torch.complex128)
    gy = torch.randn(B, Cout, H, W, dtype=torch.float64)
    gx, gw1, _ = oracle.spectral_conv2d_grads_torch(x, w1, w2, m1, m2, gy)

    def loss(xx, ww1):
        x_ft = torch.fft.rfft2(xx)
        out = torch.zeros(B, Cout, H, W // 2 + 1, dtype=torch.complex128)
        out[:, :, :m1, :m2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, :m1, :m2], ww1)
        out[:, :, -m1:, :m2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, -m1:, :m2], w2)
        return float((torch.fft.irfft2(out, s=(H, W)) * gy).sum())

    eps = 1e-6
    for idx in [(0, 1, 2, 3), (0, 0, 5, 6)]:
        e = torch.zeros_like(x)
        e[idx] = eps
        fd = (loss(x + e, w1) - loss(x - e, w1)) / (2 * eps)
        assert abs(fd - float(gx[idx])) <= 1e-6 * max(1.0, abs(fd))
    for idx in [(1, 2, 3, 1), (0, 0, 0, 0)]:
        for part in (1.0, 1j):  # d/dRe and d/dIm: torch's gradient is dL/dRe + i dL/dIm
            e = torch.zeros_like(w1)
            e[idx] = eps * part
            fd = (loss(x, w1 + e) - loss(x, w1 - e)) / (2 * eps)
            got = float(gw1[idx].real) if part == 1.0 else float(gw1[idx].imag)
            assert abs(fd - got) <= 1e-6 * max(1.0, abs(fd))


@pytest.mark.parametrize("shape", [(2, 3, 4, 20, 23, 12, 7), (1, 2, 3, 16, 16, 5, 9), (2, 3, 2, 12, 10, 4, 6)])
def test_backward_decomposition_matches_autograd(shape):
    """The sequence scx_spectral_conv2d_bwd runs, restated in numpy float64: G = forward DFT of
    grad_y (corner-1 rows that corner 2 overwrites zeroed); grad_x = inverse DFT (with its C2R
    row weights c_ky / HW) of G W^H; grad_W = ((c_ky / HW) X^H) G.  It equals autograd of the
    reference recipe, overlap, odd W and the Nyquist column included."""
    B, Cin, Cout, H, W, m1, m2 = shape
    rng = np.random.default_rng(1)
    x = rng.standard_normal((B, Cin, H, W))
    gy = rng.standard_normal((B, Cout, H, W))
    w1 = rng.standard_normal((Cin, Cout, m1, m2)) + 1j * rng.standard_normal((Cin, Cout, m1, m2))
    w2 = rng.standard_normal((Cin, Cout, m1, m2)) + 1j * rng.standard_normal((Cin, Cout, m1, m2))
    gx_ref, gw1_ref, gw2_ref = [t.numpy() for t in oracle.spectral_conv2d_grads_torch(
        torch.tensor(x), torch.tensor(w1), torch.tensor(w2), m1, m2, torch.tensor(gy))]
    rows = [np.arange(m1), np.arange(H - m1, H)]
    c = np.array([1.0 if (k == 0 or (W % 2 == 0 and k == W // 2)) else 2.0 for k in range(m2)]) / (H * W)

    def fwd(a, r):
        Fh = np.exp(-2j * np.pi * np.outer(r, np.arange(H)) / H)
        Fw = np.exp(-2j * np.pi * np.outer(np.arange(W), np.arange(m2)) / W)
        return np.einsum("rh,bchw,wk->bcrk", Fh, a, Fw)

    def inv(Y1, Y2):
        y = 0
        for Y, r, drop in ((Y1, rows[0], True), (Y2, rows[1], False)):
            keep = np.array([not (drop and v >= H - m1) for v in r])
            Gh = np.exp(2j * np.pi * np.outer(np.arange(H), r) / H) * keep
            Gw = np.exp(2j * np.pi * np.outer(np.arange(m2), np.arange(W)) / W) * c[:, None]
            y = y + np.real(np.einsum("hr,bcrk,kw->bchw", Gh, Y, Gw))
        return y

    X1, X2 = fwd(x, rows[0]), fwd(x, rows[1])
    G1, G2 = fwd(gy, rows[0]), fwd(gy, rows[1])
    if 2 * m1 > H:
        G1[:, :, H - m1:, :] = 0
    gx = inv(np.einsum("bork,iork->birk", G1, np.conj(w1)), np.einsum("bork,iork->birk", G2, np.conj(w2)))
    gw1 = np.einsum("birk,bork->iork", np.conj(X1) * c, G1)
    gw2 = np.einsum("birk,bork->iork", np.conj(X2) * c, G2)
    for ref, got in ((gx_ref, gx), (gw1_ref, gw1), (gw2_ref, gw2)):
        assert np.abs(ref - got).max() <= 1e-12 * np.abs(ref).max()


@pytest.mark.parametrize("name", ["official3d_8", "official3d_overlap"])
def test_official3d_slot_decomposition_matches_baseline(name):
    """The sequence scx_spectral_conv3d_4c_fwd runs, restated in numpy float64: forward DFTs
    keep 2 m1 / 2 m2 slot rows (low then high frequencies), the four corners are mixed, the
    slots are rebuilt with the baseline's overwrite order (a frequency held by several corners
    keeps the last corner's value, its other slots are zero), and the inverse sums over the
    slots with the C2R weights.  It equals official_baseline.py's output."""
    g = load_golden(f"conv3d_{name}.npz")
    m1, m2, m3 = (int(v) for v in g["modes"])
    x = g["x"].astype(np.float64)
    ws = [g[f"w{i}"].astype(np.complex128) for i in range(1, 5)]
    B, _, D, H, W = x.shape

    def freq(u, m, n):
        return n - 2 * m + u if u >= m else u

    f1 = np.array([freq(u, m1, D) for u in range(2 * m1)])
    f2 = np.array([freq(u, m2, H) for u in range(2 * m2)])
    Fd = np.exp(-2j * np.pi * np.outer(f1, np.arange(D)) / D)
    Fh = np.exp(-2j * np.pi * np.outer(f2, np.arange(H)) / H)
    Fw = np.exp(-2j * np.pi * np.outer(np.arange(W), np.arange(m3)) / W)
    X = np.einsum("ad,bh,icdhw,wk->icabk", Fd, Fh, x, Fw)  # [B][Cin][2 m1][2 m2][m3]
    Yall = np.zeros((B, ws[0].shape[1], 2 * m1, 2 * m2, m3), dtype=np.complex128)
    for s1 in range(2 * m1):
        for s2 in range(2 * m2):
            a, b = int(s1 >= m1), int(s2 >= m2)
            c = a + 2 * b
            kx_in = (f1[s1] < m1, f1[s1] >= D - m1)
            ky_in = (f2[s2] < m2, f2[s2] >= H - m2)
            if any(kx_in[c2 & 1] and ky_in[c2 >> 1] for c2 in range(c + 1, 4)):
                continue
            Yall[:, :, s1, s2, :] = np.einsum("bik,iok->bok", X[:, :, s1, s2, :], ws[c][:, :, s1 % m1, s2 % m2, :])
    cw = np.array([1.0 if (k == 0 or (W % 2 == 0 and k == W // 2)) else 2.0 for k in range(m3)]) / (D * H * W)
    Gd = np.exp(2j * np.pi * np.outer(np.arange(D), f1) / D)
    Gh = np.exp(2j * np.pi * np.outer(np.arange(H), f2) / H)
    Gw = np.exp(2j * np.pi * np.outer(np.arange(m3), np.arange(W)) / W) * cw[:, None]
    y = np.real(np.einsum("da,hb,ocabk,kw->ocdhw", Gd, Gh, Yall, Gw))
    fro, mx = oracle.rel_errors(g["y"], y)
    assert fro <= 1e-5 and mx <= 1e-5, (fro, mx)
