"""GPU: the NS data generator on the device and FNO-NS training with the library's forward
and backward kernels (fno_ns/train_official.py's loop, fno_model.FNO2d.forward_autograd).

* ns_vorticity_device (fp32, transforms on the library's full-spectrum DFT kernels) against
  the float64 host generator ns_vorticity on the same seed;
* forward_autograd against the reference's CPU torch path (forward(use_supa=False)), both the
  output and every parameter's gradient, and against the fused one-call forward;
* a short training run: the training loss falls and the test score is finite."""

from __future__ import annotations

import copy

import pytest
import torch

import fno_model
import fno_train
import scx_data

pytestmark = pytest.mark.gpu


def _rel(ref: torch.Tensor, got: torch.Tensor) -> float:
    ref = ref.detach().double().cpu()
    got = got.detach().double().cpu()
    return float((got - ref).norm() / ref.norm().clamp_min(1e-30))


def test_ns_generator_on_device_matches_host(cuda_device):
    host = scx_data.ns_vorticity(3, 4, 64, 64, seed=7)
    dev = scx_data.ns_vorticity_device(3, 4, 64, 64, seed=7, device=cuda_device)
    assert dev.shape == host.shape and dev.is_cuda
    for t in range(host.shape[1]):
        assert _rel(host[:, t], dev[:, t]) <= 1e-4, t


def test_ns_generator_rectangular_grid(cuda_device):
    host = scx_data.ns_vorticity(2, 2, 48, 40, seed=3)
    dev = scx_data.ns_vorticity_device(2, 2, 48, 40, seed=3, device=cuda_device)
    assert _rel(host, dev) <= 1e-4


@pytest.mark.parametrize("instance_norm", [True, False])
def test_forward_autograd_matches_cpu_path_and_grads(instance_norm, cuda_device):
    torch.manual_seed(0)
    ref = fno_model.FNO2d(modes1=12, modes2=12, width=32, n_layers=4, in_channels=10, instance_norm=instance_norm)
    dev = copy.deepcopy(ref).to(cuda_device)
    x, y = scx_data.fno_pairs_device(2, seed=5, device=cuda_device)
    pred_ref = ref(x.cpu(), use_supa=False)
    pred = dev.forward_autograd(x)
    assert _rel(pred_ref, pred) <= 1e-4
    assert _rel(dev.forward_device(x), pred) <= 1e-4
    loss_ref = torch.norm(pred_ref - y.cpu()) / torch.norm(y.cpu())
    loss = torch.norm(pred - y) / torch.norm(y)
    loss_ref.backward()
    loss.backward()
    # each gradient relative to its own norm, floored at 1e-3 of the whole model's gradient norm:
    # with InstanceNorm the lift bias has a gradient of exactly zero (a per-channel constant shift
    # of h stays constant through the spectral conv and the skip and is removed by the norm), so
    # both sides hold rounding noise there
    total = torch.sqrt(sum(p.grad.double().norm() ** 2 for p in ref.parameters())).item()
    for (name, p_ref), (_, p) in zip(ref.named_parameters(), dev.named_parameters()):
        assert p.grad is not None, name
        diff = (p.grad.detach().double().cpu() - p_ref.grad.double()).norm().item()
        scale = max(p_ref.grad.double().norm().item(), 1e-3 * total)
        assert diff <= 1e-3 * scale, (name, diff, scale)


def test_short_training_run_reduces_the_loss(cuda_device):
    torch.manual_seed(1)
    x_tr, y_tr = scx_data.fno_pairs_device(64, seed=11, device=cuda_device)
    x_te, y_te = scx_data.fno_pairs_device(16, seed=12, device=cuda_device)
    model = fno_model.FNO2d(modes1=12, modes2=12, width=32, n_layers=4, in_channels=10).to(cuda_device)
    out = fno_train.train(model, x_tr, y_tr, x_te, y_te, epochs=4, batch_size=16, lr=2e-3, seed=3,
                          scheduler=False, log=lambda s: None)
    hist = out["history"]
    assert out["steps"] == 16
    assert hist[-1]["train_l2"] < hist[0]["train_l2"]
    assert all(torch.isfinite(torch.tensor(h["test_l2"])) for h in hist)
    assert out["best_test_l2"] < 1.0
