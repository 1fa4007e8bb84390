"""FNO-2d for Navier-Stokes vorticity on B200: drop-in for fno_ns/model.py.

Same classes, constructor arguments, parameter names and construction order as
fno_ns/model.py:26-259, so ``torch.manual_seed(s); FNO2d(...)`` draws the same weights as
the reference and reference state dicts load unchanged.  Differences:

* ``SpectralConv2d.forward(x, use_supa=True)`` runs the truncated-DFT CUDA path and
  returns a tensor on x's device (host input is moved to the current CUDA device);
  ``use_supa=False`` keeps the reference's pure-torch CPU path (model.py:63-84) for
  training on the host.
* ``FNO2d.forward_supa_chain`` / ``FNO2d.forward_device`` run the whole forward on the
  device through libscx.so's fused FNO entry point (one C call per forward: lift, four
  Fourier layers, projection), optionally replayed from a CUDA graph.
* ``FNO2d.forward_autograd`` is the differentiable device forward that training uses
  (fno_train.py): spectral convolutions through the library's forward and backward kernels.
* ``instance_norm=False`` builds the norm-free layer (SpectralConv + 1x1 skip + GELU).
"""

from __future__ import annotations

import ctypes

import torch
import torch.nn as nn
import torch.nn.functional as F

import _scx
import spectral_conv_ext
from spectral_conv_ops import spectral_conv2d_autograd, spectral_conv2d_supa


def _conv1x1(conv: nn.Conv2d, x: torch.Tensor) -> torch.Tensor:
    """A 1x1 Conv2d as an fp32 channel contraction.  On CUDA, nn.Conv2d goes through cuDNN,
    which computes in TF32 by default (about 1e-3 relative error); the contraction runs as a
    cuBLAS matmul in full fp32, forward and backward."""
    out = torch.einsum("oi,bihw->bohw", conv.weight[:, :, 0, 0], x)
    return out + conv.bias[None, :, None, None] if conv.bias is not None else out


class SpectralConv2d(nn.Module):
    """fno_ns/model.py:26-84"""

    def __init__(self, in_channels: int, out_channels: int, modes1: int, modes2: int):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.modes1 = modes1
        self.modes2 = modes2
        scale = 1.0 / (in_channels * out_channels)
        self.weights1 = nn.Parameter(scale * torch.rand(in_channels, out_channels, modes1, modes2,
                                                        dtype=torch.cfloat))
        self.weights2 = nn.Parameter(scale * torch.rand(in_channels, out_channels, modes1, modes2,
                                                        dtype=torch.cfloat))

    @staticmethod
    def compl_mul2d(input_tensor: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        return torch.einsum("bixy,ioxy->boxy", input_tensor, weights)

    def forward(self, x: torch.Tensor, use_supa: bool = True) -> torch.Tensor:
        if use_supa:
            return spectral_conv2d_supa(x, self.weights1, self.weights2, self.modes1, self.modes2,
                                        use_sufft="fused", to_cpu=False)
        if x.device.type != "cpu":
            x = x.cpu()
        batch_size, _channels, height, width = x.shape
        x_ft = torch.fft.rfft2(x.to(torch.float32))
        out_ft = torch.zeros(batch_size, self.out_channels, height, width // 2 + 1, dtype=torch.complex64)
        m1, m2 = self.modes1, self.modes2
        out_ft[:, :, :m1, :m2] = self.compl_mul2d(x_ft[:, :, :m1, :m2].to(torch.complex64),
                                                  self.weights1.to(torch.complex64))
        out_ft[:, :, -m1:, :m2] = self.compl_mul2d(x_ft[:, :, -m1:, :m2].to(torch.complex64),
                                                   self.weights2.to(torch.complex64))
        return torch.fft.irfft2(out_ft, s=(height, width))


class FourierLayer(nn.Module):
    """fno_ns/model.py:87-134: spectral conv + 1x1 skip + InstanceNorm + GELU."""

    def __init__(self, width: int, modes1: int, modes2: int, instance_norm: bool = True):
        super().__init__()
        self.spectral_conv = SpectralConv2d(width, width, modes1, modes2)
        self.conv = nn.Conv2d(width, width, 1)
        self.norm = nn.InstanceNorm2d(width) if instance_norm else nn.Identity()

    def forward(self, x: torch.Tensor, use_supa: bool = True) -> torch.Tensor:
        spectral = self.spectral_conv(x, use_supa=use_supa)
        skip = self.conv(x.to(spectral.device))
        return F.gelu(self.norm(spectral + skip))

    def forward_supa(self, x: torch.Tensor, *, use_sufft="auto") -> torch.Tensor:
        """Device-resident layer (fno_ns/model.py:101-134)."""
        device = x.device
        self.conv.to(device)
        y = spectral_conv2d_supa(x, self.spectral_conv.weights1, self.spectral_conv.weights2,
                                 self.spectral_conv.modes1, self.spectral_conv.modes2, use_sufft=use_sufft,
                                 to_cpu=False)
        skip = self.conv(x)
        return F.gelu(self.norm(y + skip))


class FNO2d(nn.Module):
    """fno_ns/model.py:137-259"""

    def __init__(self, modes1: int = 12, modes2: int = 12, width: int = 32, n_layers: int = 4,
                 in_channels: int = 10, out_channels: int = 1, instance_norm: bool = True):
        super().__init__()
        if n_layers < 4:
            raise ValueError("contest requires Fourier Layer >= 4")
        if n_layers > _scx.MAX_LAYERS:
            raise ValueError(f"at most {_scx.MAX_LAYERS} Fourier layers")
        self.modes1 = modes1
        self.modes2 = modes2
        self.width = width
        self.n_layers = n_layers
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.instance_norm = instance_norm
        self.lift = nn.Conv2d(in_channels + 2, width, 1)
        self.fourier_layers = nn.ModuleList(
            [FourierLayer(width, modes1, modes2, instance_norm) for _ in range(n_layers)])
        self.project = nn.Sequential(nn.Conv2d(width, 128, 1), nn.GELU(), nn.Conv2d(128, out_channels, 1))
        self._graphs: dict = {}

    @staticmethod
    def get_grid(shape, device):
        """fno_ns/model.py:168-181"""
        batch_size, _channels, height, width = shape
        grid_x = torch.linspace(0, 1, height, device=device).reshape(1, 1, height, 1).expand(
            batch_size, 1, height, width)
        grid_y = torch.linspace(0, 1, width, device=device).reshape(1, 1, 1, width).expand(
            batch_size, 1, height, width)
        return torch.cat([grid_x, grid_y], dim=1)

    def forward(self, x: torch.Tensor, use_supa: bool = True) -> torch.Tensor:
        """fno_ns/model.py:183-198.  ``use_supa=True`` runs on the CUDA device and returns a
        host tensor like the reference; ``use_supa=False`` is the reference's CPU path."""
        if x.dim() != 4:
            raise ValueError(f"x must be [B,T,H,W], got {tuple(x.shape)}")
        if use_supa:
            return self.forward_supa_chain(x)
        x = x.to(torch.float32).cpu()
        grid = self.get_grid(x.shape, x.device)
        x = torch.cat([x, grid], dim=1)
        x = self.lift(x)
        for layer in self.fourier_layers:
            x = layer(x, use_supa=False)
        return self.project(x)

    def forward_autograd(self, x: torch.Tensor) -> torch.Tensor:
        """Differentiable forward on x's CUDA device, for training: the module's own lift,
        1x1 skips, norms, GELUs and projection run as torch ops on the device, and every
        spectral convolution runs through the library's forward and backward kernels
        (SpectralConv2dFunction), so gradients reach every parameter without a host round trip.
        Same math as forward(use_supa=False) (fno_ns/model.py:183-198)."""
        if not x.is_cuda:
            raise RuntimeError("forward_autograd needs a CUDA tensor")
        if x.dim() != 4:
            raise ValueError(f"x must be [B,T,H,W], got {tuple(x.shape)}")
        x = x.to(torch.float32)
        h = _conv1x1(self.lift, torch.cat([x, self.get_grid(x.shape, x.device)], dim=1))
        for layer in self.fourier_layers:
            sc = layer.spectral_conv
            spectral = spectral_conv2d_autograd(h.contiguous(), sc.weights1, sc.weights2, sc.modes1, sc.modes2)
            h = F.gelu(layer.norm(spectral + _conv1x1(layer.conv, h)))
        return _conv1x1(self.project[2], F.gelu(_conv1x1(self.project[0], h)))

    def prepare_supa_eval(self) -> None:
        """Moves every parameter to the current CUDA device (fno_ns/model.py:200-217)."""
        self.to(torch.device("cuda", torch.cuda.current_device()))

    # ---------------------------------------------------------------- device path

    def _device_params(self, device: torch.device):
        """(FnoParams struct, keep-alive list) pointing at device copies of the weights in
        the kernel layout (view_as_real for spectral weights, [out][in] for 1x1 convs)."""
        key = ("params", device, tuple(p._version for p in self.parameters()),
               tuple(p.data_ptr() for p in self.parameters()))
        cached = getattr(self, "_param_cache", None)
        if cached is not None and cached[0] == key:
            return cached[1], cached[2]
        keep = []

        def dev(t: torch.Tensor) -> int:
            t = t.detach().to(device)
            if t.is_complex():
                t = torch.view_as_real(t.to(torch.complex64).resolve_conj().contiguous())
            else:
                t = t.to(torch.float32).contiguous()
            keep.append(t)
            return t.data_ptr()

        p = _scx.FnoParams()
        p.lift_w = dev(self.lift.weight.reshape(self.width, -1))
        p.lift_b = dev(self.lift.bias)
        for i, layer in enumerate(self.fourier_layers):
            p.spectral_w1[i] = dev(layer.spectral_conv.weights1)
            p.spectral_w2[i] = dev(layer.spectral_conv.weights2)
            p.skip_w[i] = dev(layer.conv.weight.reshape(self.width, self.width))
            p.skip_b[i] = dev(layer.conv.bias)
        p.proj1_w = dev(self.project[0].weight.reshape(128, self.width))
        p.proj1_b = dev(self.project[0].bias)
        p.proj2_w = dev(self.project[2].weight.reshape(self.out_channels, 128))
        p.proj2_b = dev(self.project[2].bias)
        self._param_cache = (key, p, keep)
        return p, keep

    def _config(self, batch: int, height: int, width: int, channels_last: bool) -> _scx.FnoConfig:
        c = _scx.FnoConfig()
        c.batch_size = batch
        c.height = height
        c.width = width
        c.in_frames = self.in_channels
        c.input_layout = 1 if channels_last else 0
        c.hidden = self.width
        c.modes1 = self.modes1
        c.modes2 = self.modes2
        c.n_layers = self.n_layers
        c.proj_hidden = 128
        c.out_channels = self.out_channels
        c.instance_norm = 1 if self.instance_norm else 0
        return c

    def forward_device(self, x: torch.Tensor, *, channels_last: bool = False,
                       out: torch.Tensor | None = None) -> torch.Tensor:
        """Whole forward on x's CUDA device in one libscx call.

        x: [B, T, H, W] (grid channels appended inside, like the reference) or, with
        ``channels_last=True``, [B, H, W, T+2] holding the T frames then the 2 grid
        channels.  Returns [B, out_channels, H, W] on the device."""
        if not x.is_cuda:
            raise RuntimeError("forward_device needs a CUDA tensor")
        x = x.to(torch.float32).contiguous()
        if channels_last:
            B, H, W, T2 = (int(s) for s in x.shape)
            if T2 != self.in_channels + 2:
                raise ValueError(f"channels-last input needs {self.in_channels + 2} channels, got {T2}")
        else:
            B, T, H, W = (int(s) for s in x.shape)
            if T != self.in_channels:
                raise ValueError(f"x must have {self.in_channels} frames, got {T}")
        device = x.device
        params, _keep = self._device_params(device)
        cfg = self._config(B, H, W, channels_last)
        nbytes = _scx.lib.scx_fno2d_workspace_size(ctypes.byref(cfg))
        if nbytes == 0:
            raise RuntimeError("invalid FNO configuration")
        ws = spectral_conv_ext.workspace(nbytes, device)
        if out is None:
            out = torch.empty(B, self.out_channels, H, W, device=device, dtype=torch.float32)
        with _scx.device_guard(device):
            _scx.check(_scx.lib.scx_fno2d_fwd(ctypes.byref(cfg), ctypes.byref(params), x.data_ptr(),
                                              out.data_ptr(), ws.data_ptr(), ws.numel(),
                                              _scx.stream_of(device)), "scx_fno2d_fwd")
        return out

    def forward_supa_chain(self, x: torch.Tensor, *, use_sufft="auto") -> torch.Tensor:
        """fno_ns/model.py:219-259: device-resident forward, one final device-to-host copy."""
        if x.dim() != 4:
            raise ValueError(f"x must be [B,T,H,W], got {tuple(x.shape)}")
        device = x.device if x.is_cuda else torch.device("cuda", torch.cuda.current_device())
        x = x.to(device=device, dtype=torch.float32)
        return self.forward_device(x).cpu()


def count_parameters(model: nn.Module) -> int:
    return sum(parameter.numel() for parameter in model.parameters())
