"""GPU parity of the CUDA SpectralConv2d path against the oracle and the reference's
golden fixtures.  Tolerance: the reference's own 1e-4 on both metrics it uses (Frobenius
relative error, spectral_conv_combo/test_accuracy.py:16,22-27; max-abs / max|ref|,
spectral_conv_combo/test_irregular_shapes.py:78-80); the kernels compute in fp32."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import scx_data
from conftest import GOLDEN, load_golden
from oracle import oracle
from test_oracle import check_against_golden, regenerate

pytestmark = pytest.mark.gpu

TOL = 1e-4
SPECTRAL_FIXTURES = sorted(p.name for p in GOLDEN.glob("spectral_*.npz"))


def run_device(x, w1, w2, m1, m2, device):
    import spectral_conv_ops

    y = spectral_conv_ops.spectral_conv2d_supa(x.to(device), w1.to(device), w2.to(device), m1, m2,
                                               use_sufft="fused", to_cpu=False)
    torch.cuda.synchronize(device)
    return y


def assert_close(ref, got, tol=TOL):
    fro, mx = oracle.rel_errors(ref, got)
    assert fro <= tol and mx <= tol, f"frobenius rel {fro:.3e}, max-abs rel {mx:.3e}"
    return fro, mx


@pytest.mark.parametrize("fixture", SPECTRAL_FIXTURES)
def test_parity_with_reference_fixtures(fixture, cuda_device):
    g = load_golden(fixture)
    x, w1, w2, (B, Cin, Cout, H, W, m1, m2) = regenerate(g)
    y = run_device(x, w1, w2, m1, m2, cuda_device).cpu().numpy()
    assert np.isfinite(y).all()
    check_against_golden(g, y, TOL)
    ref = oracle.spectral_conv2d_torch(x, w1, w2, m1, m2).numpy()
    assert_close(ref, y)


@pytest.mark.parametrize("shape", [
    (2, 3, 4, 9, 11, 6, 6),     # 2*m1 > H (overlap), odd H and W
    (1, 2, 2, 7, 7, 7, 4),      # m1 = H, odd W, m2 = W//2+1
    (2, 3, 5, 12, 10, 4, 6),    # Nyquist column included (W even, m2 = W//2+1)
    (1, 1, 1, 1, 1, 1, 1),      # 1x1 grid
    (3, 5, 2, 16, 8, 1, 1),     # DC only
    (1, 3, 7, 33, 31, 5, 16),   # odd, Cin != Cout, B = 1
    (5, 6, 4, 40, 64, 20, 33),  # m1 = H/2 exactly, Nyquist
    (2, 4, 4, 300, 20, 3, 11),  # tall, more rows than one chunk
    (1, 2, 3, 16, 600, 8, 40),  # wide: more than one 256-column pass
])
def test_edge_shapes_vs_f64_oracle(shape, cuda_device):
    B, Cin, Cout, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(sum(shape))
    x = torch.randn(B, Cin, H, W, generator=g)
    scale = 1.0 / (Cin * Cout)
    w1 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    y = run_device(x, w1, w2, m1, m2, cuda_device).cpu().numpy()
    ref = oracle.spectral_conv2d_f64(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    assert_close(ref, y)


@pytest.mark.parametrize("name", list(scx_data.SPECTRAL_WORKLOADS))
def test_workloads_full_size(name, cuda_device):
    x, w1, w2, c = scx_data.make_spectral_case(name)
    y = run_device(x, w1, w2, c["m1"], c["m2"], cuda_device)
    ref = oracle.spectral_conv2d_torch(x, w1, w2, c["m1"], c["m2"])
    assert_close(ref.numpy(), y.cpu().numpy())


def test_linearity_full_size(cuda_device):
    """Size-independent property at the 256x256 workload: f(a x1 + b x2) = a f(x1) + b f(x2)."""
    x, w1, w2, c = scx_data.make_spectral_case("spectral_b16_c64_256x256_m32", batch=4)
    x2 = scx_data.gaussian(tuple(x.shape), 99)
    a, b = 0.75, -1.5
    y1 = run_device(x, w1, w2, c["m1"], c["m2"], cuda_device)
    y2 = run_device(x2, w1, w2, c["m1"], c["m2"], cuda_device)
    y12 = run_device(a * x + b * x2, w1, w2, c["m1"], c["m2"], cuda_device)
    # each forward carries about 1e-5 (of the output scale) of bf16x3 / fp32 rounding, and
    # a*y1 + b*y2 - y12 adds |a| + |b| + 1 = 3.25 of them
    assert_close((a * y1 + b * y2).cpu().numpy(), y12.cpu().numpy(), 3e-5)


@pytest.mark.parametrize("batch", [20, 7])  # six chunks (2, 4, 4, 4, 4, 2); ragged (1, 1, 2, 1, 1, 1)
def test_pinned_host_call_matches_device_call(batch, cuda_device):
    """A page-locked host input with a host result runs in pipelined batch chunks
    (scx_spectral_conv2d_fwd_host); every sample equals the device-resident call's result."""
    import spectral_conv_ops

    x, w1, w2, c = scx_data.make_spectral_case("spectral_b20_c32_64x64_m12", batch=batch)
    w1d, w2d = w1.to(cuda_device), w2.to(cuda_device)
    y_dev = spectral_conv_ops.spectral_conv2d_supa(x.to(cuda_device), w1d, w2d, c["m1"], c["m2"],
                                                   use_sufft="fused", to_cpu=False)
    y_host = spectral_conv_ops.spectral_conv2d_supa(x.pin_memory(), w1d, w2d, c["m1"], c["m2"],
                                                    use_sufft="fused", to_cpu=True)
    assert y_host.device.type == "cpu" and y_host.shape == y_dev.shape
    # the mixing kernel may pick another tile shape for a smaller batch (here split K over four
    # warp groups for B = 20, two for chunks of 4), which reorders its 32-term fp32 sums: about
    # 3e-6 of max|y| measured
    assert_close(y_dev.cpu().numpy(), y_host.numpy(), 1e-5)


@pytest.mark.parametrize("batch,chunks,pinned", [
    (20, 0, True), (20, 1, True), (20, 3, False), (5, 32, True), (1, 0, True), (13, 7, False)])
def test_host_entry_chunking(batch, chunks, pinned, cuda_device):
    """scx_spectral_conv2d_fwd_host for any chunk count (clamped to the batch), page-locked or
    pageable host memory: the result matches the device call sample by sample, and a second
    call into the same output gives the same bits."""
    import spectral_conv_ext

    x, w1, w2, c = scx_data.make_spectral_case("spectral_b20_c32_64x64_m12", batch=batch)
    w1d = torch.view_as_real(w1.to(cuda_device))
    w2d = torch.view_as_real(w2.to(cuda_device))
    y_dev = spectral_conv_ext.spectral_conv2d_fwd(x.to(cuda_device), w1d, w2d, c["m1"], c["m2"])
    xh = x.pin_memory() if pinned else x.contiguous()
    y_host = spectral_conv_ext.spectral_conv2d_fwd_host(xh, w1d, w2d, c["m1"], c["m2"], cuda_device,
                                                        chunks=chunks)
    assert y_host.device.type == "cpu" and y_host.shape == y_dev.shape
    # chunks may take another mixing tile shape than the whole batch (see above)
    assert_close(y_dev.cpu().numpy(), y_host.numpy(), 1e-5)
    again = torch.full_like(y_host, float("nan"))
    spectral_conv_ext.spectral_conv2d_fwd_host(xh, w1d, w2d, c["m1"], c["m2"], cuda_device, out=again,
                                               chunks=chunks)
    assert torch.equal(again, y_host)


def test_host_entry_rejects_bad_arguments(cuda_device):
    import _scx

    x, w1, w2, c = scx_data.make_spectral_case("spectral_b20_c32_64x64_m12", batch=2)
    lib = _scx.lib
    buf = torch.empty(1 << 20, dtype=torch.uint8, device=cuda_device)
    p = buf.data_ptr()
    with _scx.device_guard(cuda_device):
        # null host pointer, negative chunk count, too small a workspace
        assert lib.scx_spectral_conv2d_fwd_host(0, p, p, x.data_ptr(), 2, 32, 32, 64, 64, 12, 12, p, p, p, 1 << 20,
                                                0, None) != 0
        assert lib.scx_spectral_conv2d_fwd_host(x.data_ptr(), p, p, x.data_ptr(), 2, 32, 32, 64, 64, 12, 12, p, p,
                                                p, 1 << 20, -1, None) != 0
        assert lib.scx_spectral_conv2d_fwd_host(x.data_ptr(), p, p, x.data_ptr(), 2, 32, 32, 64, 64, 12, 12, p, p,
                                                p, 16, 0, None) != 0


def test_deterministic_and_fully_written(cuda_device):
    """Two runs are bitwise identical and every output element is written (NaN-poisoned
    output buffer)."""
    import spectral_conv_ext

    x, w1, w2, c = scx_data.make_spectral_case("spectral_b20_c32_64x64_m12")
    xd = x.to(cuda_device)
    w1d = torch.view_as_real(w1.to(cuda_device))
    w2d = torch.view_as_real(w2.to(cuda_device))
    out = torch.full((c["B"], c["Cout"], c["H"], c["W"]), float("nan"), device=cuda_device)
    y1 = spectral_conv_ext.spectral_conv2d_fwd(xd, w1d, w2d, c["m1"], c["m2"], out=out).clone()
    y2 = spectral_conv_ext.spectral_conv2d_fwd(xd, w1d, w2d, c["m1"], c["m2"])
    assert torch.isfinite(y1).all()
    assert torch.equal(y1, y2)


def test_spectral_mul_entry_points(cuda_device):
    import spectral_conv_ext
    import spectral_conv_ops

    g = torch.Generator().manual_seed(3)
    B, Cin, Cout, m1, m2 = 3, 5, 7, 6, 5
    x = torch.randn(B, Cin, m1, m2, dtype=torch.cfloat, generator=g)
    w = torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    ref = torch.einsum("bixy,ioxy->boxy", x.to(torch.complex128), w.to(torch.complex128))
    xd = torch.view_as_real(x.to(cuda_device)).contiguous()
    wd = torch.view_as_real(w.to(cuda_device)).contiguous()
    y = spectral_conv_ext.spectral_mul(xd, wd)
    assert_close(torch.view_as_real(ref).numpy(), y.cpu().numpy(), 1e-6)
    yo = torch.empty_like(y)
    spectral_conv_ext.spectral_mul_out(xd, wd, yo)
    assert torch.equal(yo, y)
    # dual: both corners in one launch
    x2 = torch.randn(B, Cin, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    x2d = torch.view_as_real(x2.to(cuda_device)).contiguous()
    w2d = torch.view_as_real(w2.to(cuda_device)).contiguous()
    y1 = torch.empty_like(y)
    y2 = torch.empty_like(y)
    spectral_conv_ext.spectral_mul_dual_out(xd, wd, x2d, w2d, y1, y2)
    ref2 = torch.einsum("bixy,ioxy->boxy", x2.to(torch.complex128), w2.to(torch.complex128))
    assert torch.equal(y1, y)
    assert_close(torch.view_as_real(ref2).numpy(), y2.cpu().numpy(), 1e-6)
    # legacy complex bridge (CPU complex out) and autograd wrapper
    yc = spectral_conv_ops.spectral_mul_supa(x, w)
    assert yc.device.type == "cpu" and yc.dtype == torch.complex64
    assert_close(torch.view_as_real(ref).numpy(), torch.view_as_real(yc).numpy(), 1e-6)


@pytest.mark.parametrize("shape", [
    (1, 3, 5, 12, 12),    # B = 1, last output-channel split ragged
    (20, 32, 36, 16, 16),  # Cout not a power of two
    (2, 4, 6, 7, 3),      # odd mode count: per-thread loads instead of TMA boxes
    (20, 32, 32, 12, 12),  # FNO layer
    (3, 64, 64, 32, 32),  # wide channels, many modes
])
def test_dual_mix_shapes(shape, cuda_device):
    """Both corners of the mode mixing against a complex128 einsum, with every output
    element written (NaN-poisoned outputs)."""
    import spectral_conv_ext

    B, Cin, Cout, m1, m2 = shape
    g = torch.Generator().manual_seed(sum(shape))
    xs = [torch.randn(B, Cin, m1, m2, dtype=torch.cfloat, generator=g) for _ in range(2)]
    ws = [torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g) for _ in range(2)]
    xd = [torch.view_as_real(t.to(cuda_device)).contiguous() for t in xs]
    wd = [torch.view_as_real(t.to(cuda_device)).contiguous() for t in ws]
    ys = [torch.full((B, Cout, m1, m2, 2), float("nan"), device=cuda_device) for _ in range(2)]
    spectral_conv_ext.spectral_mul_dual_out(xd[0], wd[0], xd[1], wd[1], ys[0], ys[1])
    for x, w, y in zip(xs, ws, ys):
        ref = torch.einsum("bixy,ioxy->boxy", x.to(torch.complex128), w.to(torch.complex128))
        assert torch.isfinite(y).all()
        assert_close(torch.view_as_real(ref).numpy(), y.cpu().numpy(), 1e-5)


@pytest.mark.parametrize("shape", [
    (16, 64, 64, 32, 32),  # the 256x256 workload's mixing: B16, C64, 1024 modes per corner
    (1, 8, 64, 3, 2),      # one batch item, one K step, 6 modes (a partial 4-mode tile)
    (7, 24, 128, 5, 4),    # odd batch, two 64-channel output blocks, 20 modes
    (8, 64, 64, 12, 12),   # N = 2B = 16 exactly
    (9, 40, 64, 4, 5),     # 2B = 18 padded to 32 columns
])
def test_tensor_core_mix_vs_einsum(shape, cuda_device):
    """The tcgen05 3xTF32 mixing (variant 9) against a complex128 einsum, every output written
    (NaN-poisoned), bitwise repeatable, and not the FFMA kernel's result (so the tensor-core
    kernel did run): both corners, then one corner."""
    import _scx
    import spectral_conv_ext

    B, Cin, Cout, m1, m2 = shape
    NM = m1 * m2
    g = torch.Generator().manual_seed(7 * sum(shape))
    xs = [torch.randn(B, Cin, m1, m2, dtype=torch.cfloat, generator=g) for _ in range(2)]
    ws = [torch.randn(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g) for _ in range(2)]
    xd = [torch.view_as_real(t.to(cuda_device)).contiguous() for t in xs]
    wd = [torch.view_as_real(t.to(cuda_device)).contiguous() for t in ws]
    lib = _scx.lib

    def run(variant):
        for nc in (1, 2):
            assert lib.scx_set_mix_variant(nc, B, Cin, Cout, NM, variant) == 0
        ys = [torch.full((B, Cout, m1, m2, 2), float("nan"), device=cuda_device) for _ in range(2)]
        spectral_conv_ext.spectral_mul_dual_out(xd[0], wd[0], xd[1], wd[1], ys[0], ys[1])
        single = spectral_conv_ext.spectral_mul(xd[1], wd[1])
        torch.cuda.synchronize(cuda_device)
        return ys, single

    try:
        ys, single = run(9)
        ys_again, _ = run(9)
        ffma, _ = run(8)  # the per-thread FFMA kernel
    finally:
        for nc in (1, 2):
            lib.scx_set_mix_variant(nc, B, Cin, Cout, NM, -1)
    for x, w, y, y2, yf in zip(xs, ws, ys, ys_again, ffma):
        ref = torch.einsum("bixy,ioxy->boxy", x.to(torch.complex128), w.to(torch.complex128))
        assert torch.isfinite(y).all()
        assert_close(torch.view_as_real(ref).numpy(), y.cpu().numpy(), 1e-5)
        assert torch.equal(y, y2)
        assert not torch.equal(y, yf)
    assert torch.equal(single, ys[1])


def test_spectral_mul_autograd_grads(cuda_device):
    """spectral_conv_combo/test_backward.py:27-54 cases."""
    import spectral_conv_ops

    for (b, ci, co, m1, m2) in [(2, 2, 3, 4, 4), (2, 4, 4, 8, 8), (2, 4, 4, 12, 12)]:
        g = torch.Generator().manual_seed(42)
        x = torch.randn(b, ci, m1, m2, generator=g, dtype=torch.cfloat)
        w = torch.randn(ci, co, m1, m2, generator=g, dtype=torch.cfloat)
        xr = x.clone().requires_grad_(True)
        wr = w.clone().requires_grad_(True)
        yr = torch.einsum("bixy,ioxy->boxy", xr, wr)
        (yr.real.pow(2) + yr.imag.pow(2)).sum().backward()
        xa = x.clone().requires_grad_(True)
        wa = w.clone().requires_grad_(True)
        ya = spectral_conv_ops.spectral_mul_autograd(xa, wa)
        (ya.real.pow(2) + ya.imag.pow(2)).sum().backward()
        for ref, got in ((yr.detach(), ya.detach()), (xr.grad, xa.grad), (wr.grad, wa.grad)):
            assert_close(torch.view_as_real(ref).numpy(), torch.view_as_real(got).numpy(), 1e-4)


@pytest.mark.parametrize("b,ci,co,m1,m2", [(20, 32, 32, 16, 16), (3, 5, 7, 6, 5), (16, 64, 48, 8, 8),
                                            (1, 9, 2, 3, 4)])
def test_spectral_mul_backward_entry_point(b, ci, co, m1, m2, cuda_device):
    """scx_spectral_mul_bwd (SpectralMulFunction's backward on the device) against the
    reference's two einsums (spectral_conv/spectral_conv_ops.py:272-278) in complex128, with
    both gradients, and each alone (bitwise the same as with both)."""
    import spectral_conv_ext

    g = torch.Generator().manual_seed(b * 1000 + ci * 10 + co)
    x = torch.randn(b, ci, m1, m2, dtype=torch.cfloat, generator=g)
    w = torch.randn(ci, co, m1, m2, dtype=torch.cfloat, generator=g)
    gy = torch.randn(b, co, m1, m2, dtype=torch.cfloat, generator=g)
    c128 = torch.complex128
    ref_x = torch.einsum("boxy,ioxy->bixy", gy.to(c128), w.to(c128).conj())
    ref_w = torch.einsum("bixy,boxy->ioxy", x.to(c128).conj(), gy.to(c128))
    xr, wr, gr = (torch.view_as_real(t).contiguous().to(cuda_device) for t in (x, w, gy))
    gx, gw = spectral_conv_ext.spectral_mul_backward(xr, wr, gr)
    torch.cuda.synchronize(cuda_device)
    assert_close(torch.view_as_real(ref_x).numpy(), gx.cpu().double().numpy())
    assert_close(torch.view_as_real(ref_w).numpy(), gw.cpu().double().numpy())
    gx_only, none_w = spectral_conv_ext.spectral_mul_backward(None, wr, gr, need_w=False)
    none_x, gw_only = spectral_conv_ext.spectral_mul_backward(xr, None, gr, need_x=False)
    assert none_w is None and none_x is None
    assert torch.equal(gx_only, gx) and torch.equal(gw_only, gw)


@pytest.mark.parametrize("H,W", [(16, 16), (9, 12), (12, 9), (64, 40), (5, 3)])
def test_full_spectrum_compat(H, W, cuda_device):
    """rfft2_sufft / irfft2_sufft compatibility entry points vs numpy FFT."""
    import spectral_conv_ext

    g = torch.Generator().manual_seed(H * 100 + W)
    x = torch.randn(2, 3, H, W, generator=g)
    xf = spectral_conv_ext.rfft2_sufft(x.to(cuda_device)).cpu()
    ref = np.fft.rfft2(x.numpy().astype(np.float64))
    got = xf[..., 0].numpy() + 1j * xf[..., 1].numpy()
    assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    spec = torch.randn(2, 3, H, W // 2 + 1, 2, generator=g)
    y = spectral_conv_ext.irfft2_sufft(spec.to(cuda_device), H, W).cpu().numpy()
    ref_y = np.fft.irfft2(spec[..., 0].numpy().astype(np.float64) + 1j * spec[..., 1].numpy(), s=(H, W))
    assert np.abs(y - ref_y).max() <= 1e-5 * np.abs(ref_y).max()
    # round trip
    back = spectral_conv_ext.irfft2_sufft(spectral_conv_ext.rfft2_sufft(x.to(cuda_device)), H, W).cpu()
    assert torch.allclose(back, x, atol=1e-5)


def test_corner_entry_points_vs_f64(cuda_device):
    import spectral_conv_ext

    g = torch.Generator().manual_seed(11)
    x = torch.randn(3, 4, 20, 18, generator=g)
    c1, c2 = spectral_conv_ext.rfft2_corners(x.to(cuda_device), 6, 7)
    r1, r2 = oracle.rfft2_corners_f64(x.numpy(), 6, 7)
    for got, ref in ((c1, r1), (c2, r2)):
        got = got.cpu().numpy()
        got = got[..., 0] + 1j * got[..., 1]
        assert np.abs(got - ref).max() <= 1e-5 * np.abs(ref).max()
    y = spectral_conv_ext.irfft2_corners(c1, c2, 20, 18).cpu().numpy()
    full = np.zeros((3, 4, 20, 10), dtype=np.complex128)
    full[:, :, :6, :7] = r1
    full[:, :, -6:, :7] = r2
    ref_y = np.fft.irfft2(full, s=(20, 18))
    assert np.abs(y - ref_y).max() <= 1e-5 * np.abs(ref_y).max()


def test_non_default_stream_and_module_api(cuda_device):
    import spectral_conv_ops

    torch.manual_seed(0)
    mod = spectral_conv_ops.SpectralConv2dSupa(6, 5, 4, 3)
    x = torch.randn(2, 6, 16, 12)
    ref = oracle.spectral_conv2d_f64(x.numpy(), mod.weights1.detach().numpy(), mod.weights2.detach().numpy(), 4, 3)
    y_host = mod(x)                      # host in, host out (reference contract)
    assert y_host.device.type == "cpu"
    assert_close(ref, y_host.detach().numpy())
    y_host2 = mod(x)
    assert y_host2.data_ptr() != y_host.data_ptr()   # no aliasing of host results
    # "auto" on a map smaller than 64 selects the reference's v1 contract: host result
    # even with to_cpu=False (spectral_conv/spectral_conv_ops.py:504-505)
    assert mod(x.to(cuda_device), to_cpu=False).device.type == "cpu"
    s = torch.cuda.Stream(cuda_device)
    with torch.cuda.stream(s):
        y_dev = mod(x.to(cuda_device), use_sufft="fused", to_cpu=False)
    s.synchronize()
    assert y_dev.is_cuda
    assert_close(ref, y_dev.cpu().detach().numpy())
    neutral = spectral_conv_ops.SpectralConv2d(6, 5, 4, 3)
    neutral.load_state_dict(mod.state_dict())
    neutral = neutral.to(cuda_device)
    assert_close(ref, neutral(x.to(cuda_device)).cpu().detach().numpy())


def test_errors_are_raised_not_faulted(cuda_device):
    import spectral_conv_ext
    import spectral_conv_ops

    x = torch.randn(1, 2, 8, 8, device=cuda_device)
    w = torch.zeros(2, 2, 9, 2, 2, device=cuda_device)
    with pytest.raises(RuntimeError):
        spectral_conv_ext.spectral_conv2d_fwd(x, w, w, 9, 2)       # m1 > H
    w = torch.zeros(2, 2, 2, 6, 2, device=cuda_device)
    with pytest.raises(RuntimeError):
        spectral_conv_ext.spectral_conv2d_fwd(x, w, w, 2, 6)       # m2 > W//2+1
    with pytest.raises(RuntimeError):
        spectral_conv_ext.spectral_mul(torch.zeros(1, 2, 2, 2, 2, device=cuda_device),
                                       torch.zeros(3, 2, 2, 2, 2, device=cuda_device))   # C_in mismatch
    with pytest.raises(ValueError):
        spectral_conv_ops.spectral_conv2d_supa(torch.zeros(2, 8, 8), w, w, 2, 2)
    # the context is still usable
    y = spectral_conv_ext.spectral_mul(torch.ones(1, 1, 1, 1, 2, device=cuda_device),
                                       torch.ones(1, 1, 1, 1, 2, device=cuda_device))
    assert y.cpu().tolist() == [[[[[0.0, 2.0]]]]]


TC_SHAPES = [
    (1, 3, 5, 64, 64, 12, 12),     # 3 planes at H=64: the last 128-row tile is half empty
    (3, 2, 2, 128, 64, 32, 24),    # 4*m1 = 128, N1 = 48
    (2, 5, 3, 128, 128, 7, 3),     # small modes, N1 = 16
    (1, 2, 2, 64, 64, 16, 16),     # N2 = W
    (4, 8, 8, 128, 128, 16, 16),
]


@pytest.mark.parametrize("shape", TC_SHAPES)
def test_tensor_core_shapes_vs_f64_oracle(shape, cuda_device):
    """Shapes routed to the tcgen05 kernels (H, W in {64, 128}) against the float64 oracle."""
    B, Cin, Cout, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(7 * sum(shape))
    x = torch.randn(B, Cin, H, W, generator=g)
    scale = 1.0 / (Cin * Cout)
    w1 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    y = run_device(x, w1, w2, m1, m2, cuda_device).cpu().numpy()
    ref = oracle.spectral_conv2d_f64(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    assert_close(ref, y)


def test_tensor_core_corners_vs_f64(cuda_device):
    """The tcgen05 forward alone: corner spectra against the float64 direct DFT."""
    import spectral_conv_ext

    g = torch.Generator().manual_seed(12)
    x = torch.randn(3, 4, 64, 64, generator=g)
    c1, c2 = spectral_conv_ext.rfft2_corners(x.to(cuda_device), 12, 12)
    r1, r2 = oracle.rfft2_corners_f64(x.numpy(), 12, 12)
    for got, ref in ((c1, r1), (c2, r2)):
        got = got.cpu().numpy()
        got = got[..., 0] + 1j * got[..., 1]
        assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()
    y = spectral_conv_ext.irfft2_corners(c1, c2, 64, 64).cpu().numpy()
    full = np.zeros((3, 4, 64, 33), dtype=np.complex128)
    full[:, :, :12, :12] = r1
    full[:, :, -12:, :12] = r2
    ref_y = np.fft.irfft2(full, s=(64, 64))
    assert np.abs(y - ref_y).max() <= 1e-4 * np.abs(ref_y).max()


FWD_TC_SHAPES = [
    (1, 3, 64, 64, 12, 12),      # W = 64: 2 planes per column tile, the last one half empty
    (1, 1, 128, 128, 16, 16),    # one plane: fewer planes than SMs
    (2, 5, 128, 64, 16, 24),     # H != W, 24 columns per TW block
    (3, 3, 64, 128, 5, 32),      # m2 = 32, slots of the second group unused
    (4, 8, 128, 128, 7, 3),      # 8 columns per TW block
    (40, 32, 128, 128, 16, 16),  # several 2-plane tiles per CTA
    (2, 151, 64, 64, 12, 12),    # odd plane count over all SMs
    # folded: one launch, CTAs in parity groups of four, the quadrants combined in the converters
    (2, 3, 256, 256, 32, 32),    # 128 x 128 parity sub-planes
    (1, 5, 128, 256, 16, 20),    # 64 x 128 sub-planes
    (3, 2, 256, 128, 16, 16),    # 128 x 64 sub-planes: two planes per column tile
    (2, 2, 128, 128, 24, 20),    # 2*m1 > 32 at 128: 64 x 64 sub-planes
    (1, 1, 256, 256, 8, 12),     # one plane: most CTA groups have nothing to do
]


@pytest.mark.parametrize("shape", FWD_TC_SHAPES)
def test_forward_corners_vs_f64(shape, cuda_device):
    """Corner spectra of the forward transform against the float64 direct DFT."""
    import spectral_conv_ext

    B, C, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(3 * sum(shape))
    x = torch.randn(B, C, H, W, generator=g)
    xd = x.to(cuda_device)
    c1, c2 = spectral_conv_ext.rfft2_corners(xd, m1, m2)
    r1, r2 = oracle.rfft2_corners_f64(x.numpy(), m1, m2)
    for got, ref in ((c1, r1), (c2, r2)):
        got = got.cpu().numpy()
        got = got[..., 0] + 1j * got[..., 1]
        err = np.abs(got - ref).max() / np.abs(ref).max()
        assert err <= 2e-5, err
    # the pipelined kernel is race-free: repeated runs agree bit for bit
    for _ in range(3):
        d1, d2 = spectral_conv_ext.rfft2_corners(xd, m1, m2)
        assert torch.equal(d1, c1) and torch.equal(d2, c2)


INV_TC_SHAPES = [
    (1, 3, 64, 64, 12, 12),      # 2 planes per S5 chain, the last group mostly empty
    (1, 1, 128, 128, 16, 16),    # one plane
    (2, 5, 128, 64, 16, 24),     # H != W, 64 spectrum rows per plane
    (3, 3, 64, 128, 5, 32),      # m2 = 32
    (4, 8, 128, 128, 7, 3),
    (40, 32, 128, 128, 16, 16),  # several groups per CTA
    (2, 151, 64, 64, 12, 12),    # odd plane count over all SMs
    # 256 x 256: four CTAs per plane group, one per output quadrant, from the full corners
    (2, 3, 256, 256, 32, 32),    # 64 spectrum rows, 32 columns
    (1, 5, 256, 256, 16, 20),
    (3, 7, 256, 256, 7, 3),      # odd plane count: a partial last group
    (1, 1, 256, 256, 1, 1),      # DC only, one plane
]


@pytest.mark.parametrize("shape", INV_TC_SHAPES)
def test_inverse_corners_vs_f64(shape, cuda_device):
    """Zero-padded inverse from the two corner spectra against numpy's float64 irfft2."""
    import spectral_conv_ext

    B, C, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(5 * sum(shape))
    c1 = torch.randn(B, C, m1, m2, 2, generator=g)
    c2 = torch.randn(B, C, m1, m2, 2, generator=g)
    c1d, c2d = c1.to(cuda_device), c2.to(cuda_device)
    yd = spectral_conv_ext.irfft2_corners(c1d, c2d, H, W)
    for _ in range(3):  # repeated runs agree bit for bit
        assert torch.equal(spectral_conv_ext.irfft2_corners(c1d, c2d, H, W), yd)
    y = yd.cpu().numpy()
    full = np.zeros((B, C, H, W // 2 + 1), dtype=np.complex128)
    full[:, :, :m1, :m2] = c1[..., 0].numpy() + 1j * c1[..., 1].numpy()
    full[:, :, H - m1:, :m2] = c2[..., 0].numpy() + 1j * c2[..., 1].numpy()
    ref = np.fft.irfft2(full, s=(H, W))
    err = np.abs(y - ref).max() / np.abs(ref).max()
    assert err <= 2e-5, err


@pytest.mark.parametrize("shape", [
    (2, 3, 4, 256, 256, 8, 12),    # folded tensor-core path, small modes
    (1, 2, 2, 256, 256, 32, 64),   # m1 = 32, m2 = 64: 16 slots and 32 columns per parity class
    (2, 2, 3, 128, 128, 24, 20),   # 2*m1 > 32 at 128: folded into 64 x 64 sub-planes
    (3, 4, 2, 256, 128, 16, 16),   # non-square folded plane
    (2, 3, 3, 128, 256, 16, 20),   # non-square, the other way
])
def test_folded_path_vs_f64_oracle(shape, cuda_device):
    """Planes folded into four parity sub-planes (fused forward with its workspace)."""
    B, Cin, Cout, H, W, m1, m2 = shape
    g = torch.Generator().manual_seed(sum(shape) + 1)
    x = torch.randn(B, Cin, H, W, generator=g)
    scale = 1.0 / (Cin * Cout)
    w1 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    w2 = scale * torch.rand(Cin, Cout, m1, m2, dtype=torch.cfloat, generator=g)
    y = run_device(x, w1, w2, m1, m2, cuda_device).cpu().numpy()
    ref = oracle.spectral_conv2d_f64(x.numpy(), w1.numpy(), w2.numpy(), m1, m2)
    assert_close(ref, y)


def test_zz_watchdog_clean(cuda_device):
    """No tensor-core kernel gave up on a wait during this session."""
    import _scx

    torch.cuda.synchronize(cuda_device)
    assert _scx.lib.scx_watchdog(0) == 0
