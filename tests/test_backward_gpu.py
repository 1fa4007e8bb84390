"""GPU parity of the SpectralConv2d backward (scx_spectral_conv2d_bwd) against torch autograd
of the reference recipe (spectral_conv/reference_pytorch.py:30-47) in float64 on the CPU.
The reference's own backward test (test_backward.py:27-54) checks SpectralMulFunction the
same way, against autograd of the einsum; tolerance here is the reference's 1e-4 on the
Frobenius and max-abs relative errors."""

from __future__ import annotations

import pytest
import torch

import scx_data
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4

SHAPES = [
    # B, Cin, Cout, H, W, m1, m2
    (3, 16, 24, 64, 64, 12, 12),     # 64x64 tensor-core path
    (2, 32, 32, 128, 128, 16, 16),   # the headline shape, fewer items
    (2, 8, 8, 20, 23, 12, 7),        # corners overlap (2 m1 > H), odd W
    (1, 4, 6, 16, 16, 5, 9),         # Nyquist column kept (m2 = W/2 + 1)
    (1, 16, 16, 256, 256, 32, 32),   # folded 256x256 path
]


def _close(ref, got, what):
    fro, mx = oracle.rel_errors(ref.detach().cpu().numpy(), got.detach().cpu().numpy())
    assert fro <= TOL and mx <= TOL, f"{what}: frobenius rel {fro:.3e}, max-abs rel {mx:.3e}"


def _case(shape, seed):
    B, Cin, Cout, H, W, m1, m2 = shape
    x = scx_data.gaussian((B, Cin, H, W), seed)
    w1, w2 = scx_data.spectral_weights(Cin, Cout, m1, m2, seed + 1)
    gy = scx_data.gaussian((B, Cout, H, W), seed + 2)
    return x, w1, w2, gy


@pytest.mark.parametrize("shape", SHAPES, ids=lambda s: "x".join(map(str, s)))
def test_backward_matches_autograd_of_reference(shape, cuda_device):
    import spectral_conv_ops

    B, Cin, Cout, H, W, m1, m2 = shape
    x, w1, w2, gy = _case(shape, 40)
    gx_ref, gw1_ref, gw2_ref = oracle.spectral_conv2d_grads_torch(x, w1, w2, m1, m2, gy)
    xd = x.to(cuda_device).requires_grad_(True)
    w1d = w1.to(cuda_device).requires_grad_(True)
    w2d = w2.to(cuda_device).requires_grad_(True)
    y = spectral_conv_ops.spectral_conv2d_autograd(xd, w1d, w2d, m1, m2)
    y.backward(gy.to(cuda_device))
    _close(gx_ref, xd.grad, "grad_x")
    _close(torch.view_as_real(gw1_ref), torch.view_as_real(w1d.grad), "grad_w1")
    _close(torch.view_as_real(gw2_ref), torch.view_as_real(w2d.grad), "grad_w2")
    assert w1d.grad.dtype == torch.complex64 and xd.grad.dtype == torch.float32


def test_module_training_step_and_partial_grads(cuda_device):
    """SpectralConv2d (the state-dict twin of reference_pytorch.SpectralConv2d) trains on the
    device: a loss's gradients match the oracle; with frozen weights only grad_x is made, and
    with a constant input only the weight gradients."""
    import spectral_conv_ops

    shape = (2, 8, 12, 32, 32, 6, 6)
    B, Cin, Cout, H, W, m1, m2 = shape
    x, _, _, gy = _case(shape, 50)
    torch.manual_seed(3)
    mod = spectral_conv_ops.SpectralConv2d(Cin, Cout, m1, m2).to(cuda_device)
    gx_ref, gw1_ref, gw2_ref = oracle.spectral_conv2d_grads_torch(x, mod.weights1.detach().cpu(),
                                                                  mod.weights2.detach().cpu(), m1, m2, gy)
    y = mod(x.to(cuda_device))
    (y * gy.to(cuda_device)).sum().backward()
    _close(torch.view_as_real(gw1_ref), torch.view_as_real(mod.weights1.grad), "module grad_w1")
    _close(torch.view_as_real(gw2_ref), torch.view_as_real(mod.weights2.grad), "module grad_w2")

    mod.zero_grad(set_to_none=True)
    mod.requires_grad_(False)
    xd = x.to(cuda_device).requires_grad_(True)
    mod(xd).backward(gy.to(cuda_device))
    _close(gx_ref, xd.grad, "frozen-weight grad_x")
    assert mod.weights1.grad is None

    mod.requires_grad_(True)
    mod(x.to(cuda_device)).backward(gy.to(cuda_device))
    _close(torch.view_as_real(gw1_ref), torch.view_as_real(mod.weights1.grad), "constant-input grad_w1")


def test_backward_is_deterministic(cuda_device):
    import spectral_conv_ext

    shape = (3, 16, 24, 64, 64, 12, 12)
    B, Cin, Cout, H, W, m1, m2 = shape
    x, w1, w2, gy = _case(shape, 60)
    w1d = torch.view_as_real(w1.to(cuda_device))
    w2d = torch.view_as_real(w2.to(cuda_device))
    _, xc = spectral_conv_ext.spectral_conv2d_fwd_saved(x.to(cuda_device), w1d, w2d, m1, m2)
    a = spectral_conv_ext.spectral_conv2d_bwd(gy.to(cuda_device), xc, w1d, w2d, m1, m2)
    b = spectral_conv_ext.spectral_conv2d_bwd(gy.to(cuda_device), xc, w1d, w2d, m1, m2)
    for u, v in zip(a, b):
        assert torch.equal(u, v)
