"""Seeded synthetic inputs for the SpectralConv2d / FNO-NS workloads.

The public FNO Navier-Stokes data is not available offline, so fields with the same
shapes and spectra stand in for it.  Every generator runs on the CPU with an explicit
``torch.Generator`` so that the device path and the CPU oracle see identical bytes.

* ``gaussian``           x ~ N(0, 1)
* ``spectral_weights``   (1/(Cin*Cout)) * U[0,1) real and imaginary parts, the init of
                         spectral_conv/reference_pytorch.py:19-25
* ``grf``                Gaussian random field with power spectrum (k^2 + tau^2)^-alpha,
                         each field normalised to unit variance
* ``ns_vorticity``       GRF initial vorticity (spectrum (k^2+49)^-2.5) advanced by a
                         pseudo-spectral 2-D Navier-Stokes vorticity step (nu, dt)
* ``ns_vorticity_device`` the same on a CUDA device, transforms on the library's DFT kernels
* ``fno_pairs_device``   (10 frames, next frame) training pairs from it
* ``fno_input``          [B, H, W, T+2] channels-last: T vorticity frames + 2 grid channels
"""

from __future__ import annotations

import math

import torch


def _gen(seed: int) -> torch.Generator:
    g = torch.Generator(device="cpu")
    g.manual_seed(int(seed))
    return g


def gaussian(shape, seed: int) -> torch.Tensor:
    return torch.randn(*shape, generator=_gen(seed), dtype=torch.float32)


def spectral_weights(cin: int, cout: int, m1: int, m2: int, seed: int):
    """Two complex64 weight tensors [Cin, Cout, m1, m2] with the reference's init."""
    g = _gen(seed)
    scale = 1.0 / (cin * cout)
    w1 = scale * torch.rand(cin, cout, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = scale * torch.rand(cin, cout, m1, m2, dtype=torch.cfloat, generator=g)
    return w1, w2


def _wavenumber_sq(H: int, W: int) -> torch.Tensor:
    kx = torch.fft.fftfreq(H, d=1.0 / H).to(torch.float64)
    ky = torch.fft.rfftfreq(W, d=1.0 / W).to(torch.float64)
    return kx[:, None] ** 2 + ky[None, :] ** 2


def grf(shape, seed: int, *, alpha: float = 2.0, tau: float = 3.0) -> torch.Tensor:
    """GRF with power spectrum (k^2 + tau^2)^-alpha over integer wavenumbers k."""
    *lead, H, W = shape
    noise = torch.randn(*lead, H, W, generator=_gen(seed), dtype=torch.float64)
    spec = torch.fft.rfft2(noise)
    amp = (_wavenumber_sq(H, W) + tau * tau) ** (-alpha / 2.0)
    amp[0, 0] = 0.0
    field = torch.fft.irfft2(spec * amp, s=(H, W))
    field = field - field.mean(dim=(-2, -1), keepdim=True)
    field = field / field.std(dim=(-2, -1), keepdim=True).clamp_min(1e-30)
    return field.to(torch.float32)


def ns_vorticity(batch: int, frames: int, H: int, W: int, seed: int, *, nu: float = 1e-3,
                 dt: float = 1e-4, substeps: int = 1) -> torch.Tensor:
    """[batch, frames, H, W] vorticity: GRF initial state (spectrum (k^2+49)^-2.5)
    advanced on the unit torus by a pseudo-spectral step of
        w_t + u . grad(w) = nu * lap(w) + f,   u = (psi_y, -psi_x),  -lap(psi) = w
    with Crank-Nicolson diffusion, explicit advection, 2/3-rule dealiasing and the
    forcing f = 0.1 (sin 2pi(x+y) + cos 2pi(x+y)).  One frame every ``substeps`` steps."""
    w = grf((batch, H, W), seed, alpha=2.5, tau=7.0).to(torch.float64)
    kx = torch.fft.fftfreq(H, d=1.0 / H).to(torch.float64)[:, None].expand(H, W // 2 + 1)
    ky = torch.fft.rfftfreq(W, d=1.0 / W).to(torch.float64)[None, :].expand(H, W // 2 + 1)
    k2 = 4.0 * math.pi ** 2 * (kx ** 2 + ky ** 2)
    k2_inv = torch.where(k2 > 0, 1.0 / k2.clamp_min(1e-30), torch.zeros_like(k2))
    dealias = ((kx.abs() <= (2.0 / 3.0) * (H // 2)) & (ky.abs() <= (2.0 / 3.0) * (W // 2))).to(torch.float64)
    xs = torch.linspace(0, 1, H + 1, dtype=torch.float64)[:-1]
    ys = torch.linspace(0, 1, W + 1, dtype=torch.float64)[:-1]
    X, Y = torch.meshgrid(xs, ys, indexing="ij")
    f_hat = torch.fft.rfft2(0.1 * (torch.sin(2 * math.pi * (X + Y)) + torch.cos(2 * math.pi * (X + Y))))
    w_hat = torch.fft.rfft2(w)
    out = torch.empty(batch, frames, H, W, dtype=torch.float32)
    for t in range(frames):
        for _ in range(substeps):
            psi_hat = w_hat * k2_inv
            u = torch.fft.irfft2(2j * math.pi * ky * psi_hat, s=(H, W))
            v = torch.fft.irfft2(-2j * math.pi * kx * psi_hat, s=(H, W))
            wx = torch.fft.irfft2(2j * math.pi * kx * w_hat, s=(H, W))
            wy = torch.fft.irfft2(2j * math.pi * ky * w_hat, s=(H, W))
            adv_hat = torch.fft.rfft2(u * wx + v * wy) * dealias
            w_hat = ((1.0 - 0.5 * dt * nu * k2) * w_hat + dt * (f_hat - adv_hat)) / (1.0 + 0.5 * dt * nu * k2)
        out[:, t] = torch.fft.irfft2(w_hat, s=(H, W)).to(torch.float32)
    return out


def ns_vorticity_device(batch: int, frames: int, H: int, W: int, seed: int, device, *, nu: float = 1e-3,
                        dt: float = 1e-4, substeps: int = 1) -> torch.Tensor:
    """``ns_vorticity`` on a CUDA device, in fp32: the same initial field (the GRF noise is
    drawn on the host from the same seed) and the same pseudo-spectral step, with every
    transform on the library's own full-spectrum DFT kernels (``spectral_conv_ext.rfft2_sufft``
    / ``irfft2_sufft``, no torch.fft) and the spectral products as device tensor arithmetic.
    Per step the four fields u, v, w_x, w_y go through one batched inverse transform."""
    import spectral_conv_ext as ext

    def rfft2(f):  # [n, H, W] real -> [n, H, W/2+1] complex
        return torch.view_as_complex(ext.rfft2_sufft(f.unsqueeze(1).contiguous())[:, 0])

    def irfft2(fh):  # [n, C, H, W/2+1] complex -> [n, C, H, W] real
        return ext.irfft2_sufft(torch.view_as_real(fh).contiguous(), H, W)

    noise = torch.randn(batch, H, W, generator=_gen(seed), dtype=torch.float64).to(torch.float32).to(device)
    amp = ((_wavenumber_sq(H, W) + 49.0) ** (-2.5 / 2.0))
    amp[0, 0] = 0.0
    field = irfft2((rfft2(noise) * amp.to(torch.float32).to(device)).unsqueeze(1))[:, 0]
    field = field - field.mean(dim=(-2, -1), keepdim=True)
    w = field / field.std(dim=(-2, -1), keepdim=True).clamp_min(1e-30)
    Wf = W // 2 + 1
    kx = torch.fft.fftfreq(H, d=1.0 / H).to(torch.float32)[:, None].expand(H, Wf).to(device)
    ky = torch.fft.rfftfreq(W, d=1.0 / W).to(torch.float32)[None, :].expand(H, Wf).to(device)
    two_pi = 2.0 * math.pi
    k2 = (two_pi ** 2) * (kx ** 2 + ky ** 2)
    k2_inv = torch.where(k2 > 0, 1.0 / k2.clamp_min(1e-30), torch.zeros_like(k2))
    dealias = ((kx.abs() <= (2.0 / 3.0) * (H // 2)) & (ky.abs() <= (2.0 / 3.0) * (W // 2))).to(torch.float32)
    xs = torch.linspace(0, 1, H + 1, dtype=torch.float64)[:-1]
    ys = torch.linspace(0, 1, W + 1, dtype=torch.float64)[:-1]
    X, Y = torch.meshgrid(xs, ys, indexing="ij")
    forcing = (0.1 * (torch.sin(two_pi * (X + Y)) + torch.cos(two_pi * (X + Y)))).to(torch.float32).to(device)
    f_hat = rfft2(forcing.unsqueeze(0))[0]
    ikx, iky = (1j * two_pi) * kx, (1j * two_pi) * ky
    lhs = 1.0 + 0.5 * dt * nu * k2
    rhs = 1.0 - 0.5 * dt * nu * k2
    w_hat = rfft2(w)
    out = torch.empty(batch, frames, H, W, device=device, dtype=torch.float32)
    for t in range(frames):
        for _ in range(substeps):
            psi_hat = w_hat * k2_inv
            fields = irfft2(torch.stack([iky * psi_hat, -ikx * psi_hat, ikx * w_hat, iky * w_hat], dim=1))
            u, v, wx, wy = fields.unbind(1)
            adv_hat = rfft2(u * wx + v * wy) * dealias
            w_hat = (rhs * w_hat + dt * (f_hat - adv_hat)) / lhs
        out[:, t] = irfft2(w_hat.unsqueeze(1))[:, 0]
    return out


def fno_pairs_device(n: int, seed: int, device, *, H: int = 64, W: int = 64, frames_in: int = 10):
    """(x [n, frames_in, H, W], y [n, 1, H, W]) on the device: ``frames_in`` vorticity frames
    and the next one as the target (the input/target split of fno_ns/dataset.py's sequence
    dataset), from ``ns_vorticity_device``."""
    seq = ns_vorticity_device(n, frames_in + 1, H, W, seed, device)
    return seq[:, :frames_in].contiguous(), seq[:, frames_in:].contiguous()


def grid_channels(batch: int, H: int, W: int) -> torch.Tensor:
    """[B, 2, H, W]: linspace(0,1,H) down the rows and linspace(0,1,W) along the columns,
    the grid of fno_ns/model.py:168-181."""
    gx = torch.linspace(0, 1, H).reshape(1, 1, H, 1).expand(batch, 1, H, W)
    gy = torch.linspace(0, 1, W).reshape(1, 1, 1, W).expand(batch, 1, H, W)
    return torch.cat([gx, gy], dim=1)


def fno_input(batch: int, seed: int, *, H: int = 64, W: int = 64, frames: int = 10) -> torch.Tensor:
    """[B, H, W, frames + 2] channels-last FNO-NS input (vorticity frames then grid)."""
    vort = ns_vorticity(batch, frames, H, W, seed)
    full = torch.cat([vort, grid_channels(batch, H, W)], dim=1)
    return full.permute(0, 2, 3, 1).contiguous()


# ---------------------------------------------------------------------------------------
# Named workloads (sizes in the name).  ``input``: "gaussian" or "grf"; weights use seed+1000.
SPECTRAL_WORKLOADS = {
    "spectral_b20_c32_64x64_m12": dict(B=20, Cin=32, Cout=32, H=64, W=64, m1=12, m2=12,
                                       input="gaussian", seed=1),
    "spectral_b20_c32_128x128_m16_grf": dict(B=20, Cin=32, Cout=32, H=128, W=128, m1=16, m2=16,
                                             input="grf", seed=2),
    "spectral_b16_c64_256x256_m32": dict(B=16, Cin=64, Cout=64, H=256, W=256, m1=32, m2=32,
                                         input="gaussian", seed=3),
    "spectral_b7_c20to36_96x160_m16x20": dict(B=7, Cin=20, Cout=36, H=96, W=160, m1=16, m2=20,
                                              input="gaussian", seed=4),
    "spectral_b3_c24_100x72_m10": dict(B=3, Cin=24, Cout=24, H=100, W=72, m1=10, m2=10,
                                       input="gaussian", seed=5),
    "spectral_b1_c48_130x130_m24": dict(B=1, Cin=48, Cout=48, H=130, W=130, m1=24, m2=24,
                                        input="gaussian", seed=6),
}

FNO_WORKLOAD = dict(name="fno_ns_b20_w32_64x64_m12_l4", B=20, H=64, W=64, frames=10, width=32,
                    modes=12, layers=4, seed=7, init_seed=0)


def make_spectral_case(name: str, batch: int | None = None):
    """(x [B,Cin,H,W] float32, w1, w2 complex64 [Cin,Cout,m1,m2], cfg) for a named workload.
    ``batch`` overrides B (the first ``batch`` items are identical to the full case)."""
    cfg = dict(SPECTRAL_WORKLOADS[name])
    if batch is not None:
        cfg["B"] = batch
    full_b = SPECTRAL_WORKLOADS[name]["B"]
    shape = (max(full_b, cfg["B"]), cfg["Cin"], cfg["H"], cfg["W"])
    if cfg["input"] == "grf":
        x = grf(shape, cfg["seed"], alpha=2.0, tau=3.0)
    else:
        x = gaussian(shape, cfg["seed"])
    x = x[: cfg["B"]].contiguous()
    w1, w2 = spectral_weights(cfg["Cin"], cfg["Cout"], cfg["m1"], cfg["m2"], cfg["seed"] + 1000)
    return x, w1, w2, cfg


def reference_accuracy_case(batch, cin, cout, H, W, m1, m2, seed):
    """Inputs of spectral_conv_combo/test_accuracy.py:30-33: torch.manual_seed(seed), the
    module's two torch.rand weights, then x = torch.randn."""
    torch.manual_seed(seed)
    scale = 1.0 / (cin * cout)
    w1 = scale * torch.rand(cin, cout, m1, m2, dtype=torch.cfloat)
    w2 = scale * torch.rand(cin, cout, m1, m2, dtype=torch.cfloat)
    x = torch.randn(batch, cin, H, W, dtype=torch.float32)
    return x, w1, w2


def reference_irregular_case(batch, cin, H, W, cout=64, modes=16):
    """Inputs of spectral_conv_combo/test_irregular_shapes.py:154-163 (seed 0, M = min(16,
    min(H,W)//2)); returns (x, w1, w2, M)."""
    M = min(modes, min(H, W) // 2)
    torch.manual_seed(0)
    x = torch.randn(batch, cin, H, W, dtype=torch.float32)
    scale = 1.0 / (cin * cout)
    w1 = (scale * torch.rand(cin, cout, M, M, dtype=torch.cfloat)).contiguous()
    w2 = (scale * torch.rand(cin, cout, M, M, dtype=torch.cfloat)).contiguous()
    return x, w1, w2, M


# spectral_conv_combo/test_accuracy.py:61-65 (name, B, Cin, Cout, H, W, m1, m2, seed)
REFERENCE_ACCURACY_CASES = [
    ("tiny_8x8", 2, 2, 3, 8, 8, 2, 2, 11),
    ("small_32x32", 2, 4, 4, 32, 32, 8, 8, 22),
    ("target_64x64", 2, 4, 4, 64, 64, 12, 12, 33),
    ("official_128", 4, 32, 64, 128, 128, 16, 16, 44),
    ("official_256_fused", 4, 32, 64, 256, 256, 16, 16, 55),
]

# spectral_conv_combo/test_irregular_shapes.py:22-32 (B, Cin, H, W); Cout = 64
REFERENCE_IRREGULAR_SHAPES = [
    (4, 32, 64, 40), (4, 32, 40, 64), (4, 32, 48, 48), (4, 32, 72, 72), (4, 32, 96, 96),
    (4, 32, 160, 160), (4, 32, 192, 192), (4, 32, 256, 64), (2, 16, 100, 100),
]


# spectral_conv_combo/test_3d_accuracy.py:69-72 (name, B, Cin, Cout, D, H, W, (m1, m2, m3), seed)
REFERENCE_3D_CASES = [
    ("tiny_8", 2, 2, 3, 8, 8, 8, (2, 2, 2), 11),
    ("small_16", 2, 4, 4, 16, 16, 16, (4, 4, 4), 22),
]


def reference_3d_case(batch, cin, cout, D, H, W, modes, seed):
    """The input and weights test_3d_accuracy.py:40-43 draws: x ~ N(0,1) from a generator
    seeded with ``seed``; weights with real then imaginary parts uniform in [-0.5, 0.5) from a
    generator seeded with ``seed + 1`` (reference_pytorch.py:85-102), drawn as
    [Cin, Cout, m1, m2*m3] and reshaped to [Cin, Cout, m1, m2, m3]."""
    x = torch.randn(batch, cin, D, H, W, generator=_gen(seed))
    g = _gen(seed + 1)
    m1, m2, m3 = modes
    re = torch.empty(cin, cout, m1, m2 * m3, dtype=torch.float32).uniform_(-0.5, 0.5, generator=g)
    im = torch.empty_like(re).uniform_(-0.5, 0.5, generator=g)
    w = torch.complex(re, im).reshape(cin, cout, m1, m2, m3)
    return x, w


# Four-corner SpectralConv3d (official_baseline.py:60-100) fixture cases:
# (name, B, Cin, Cout, D, H, W, (m1, m2, m3), seed); the module is initialised after
# torch.manual_seed(seed), the input drawn from a generator seeded with seed + 1.
OFFICIAL_3D_CASES = [
    ("official3d_8", 2, 3, 4, 8, 8, 8, (3, 3, 3), 31),
    ("official3d_overlap", 1, 2, 3, 6, 10, 12, (4, 6, 7), 32),  # 2 m1 > D, 2 m2 > H, Nyquist
]
