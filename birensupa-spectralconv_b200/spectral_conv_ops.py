"""Drop-in for the reference's ``spectral_conv_ops`` (spectral_conv/spectral_conv_ops.py,
spectral_conv_combo/spectral_conv_ops.py) on B200.

Same public names, signatures and error behaviour.  Every path runs on the CUDA device
through libscx.so (truncated forward DFT -> dual-corner mixing -> zero-padded inverse
DFT); there is no CPU FFT path and no CPU fallback.  ``use_sufft`` is still validated
exactly like the reference's ``resolve_use_sufft`` but only decides the return device
contract of the old ``v1`` path (host tensor), never where the math runs.

Reference defects that are fixed here, not replicated:
* the host result of ``to_cpu=True`` is a fresh tensor, not a shared staging buffer that
  the next call overwrites (spectral_conv_combo/spectral_conv_ops.py:426-431);
* device weights are used in place (``view_as_real``), so ``.detach()`` no longer defeats
  a cache (spectral_conv/spectral_conv_ops.py:155-188); host weights are uploaded once
  per (Parameter, version) or per content.
"""

from __future__ import annotations

import hashlib
import weakref

import torch
import torch.nn as nn

import scx_tune
import spectral_conv_ext

# Kernel variants measured per shape by scx_tune.py, when a table has been saved
# ($SCX_TUNE_TABLE, else the package's tune_table.json): applied once, at import.
TUNED_VARIANTS = scx_tune.load()
_WEIGHT_DEVICE_CACHE: dict[tuple, torch.Tensor] = {}
_PARAM_CACHE: dict[tuple, tuple] = {}
_WEIGHT_CACHE_MAX = 64

# Per-shape decisions, same shape and meaning as the reference's table
# (spectral_conv_combo/spectral_conv_ops.py:45-63).  Empty by default.
_AUTO_TUNE_TABLE: dict = {}
_AUTO_TUNE_DEFAULTS: dict = {"use_sufft": "auto", "buffer_max": 4, "fused_block": None}


def _device_for(x: torch.Tensor) -> torch.device:
    if x.is_cuda:
        return x.device
    if not torch.cuda.is_available():
        raise RuntimeError("spectral_conv_ops needs a CUDA device (there is no CPU path)")
    return torch.device("cuda", torch.cuda.current_device())


def _complex_to_interleaved(tensor_complex: torch.Tensor) -> torch.Tensor:
    tensor_complex = tensor_complex.to(torch.complex64).resolve_conj().contiguous()
    return torch.view_as_real(tensor_complex).contiguous()


def _interleaved_to_complex(tensor_real_imag: torch.Tensor) -> torch.Tensor:
    return torch.view_as_complex(tensor_real_imag.contiguous())


def _weights_to_device_cached(weights: torch.Tensor, device: torch.device) -> torch.Tensor:
    """Interleaved float32 [Cin,Cout,m1,m2,2] weights on ``device``.

    A complex64 contiguous tensor already on the device is viewed in place (no copy, no
    cache).  Anything else is converted once and cached: Parameters by identity and
    ``_version`` (like spectral_conv/spectral_conv_ops.py:161-177), other tensors by a
    content hash (:179-188)."""
    w = weights.detach()
    if w.device == device and w.dtype == torch.complex64 and w.is_contiguous() and not w.is_conj():
        return torch.view_as_real(w)
    if w.device == device and w.dtype == torch.float32 and w.dim() == 5 and w.is_contiguous():
        return w
    if isinstance(weights, nn.Parameter):
        key = (id(weights), str(device))
        version = int(getattr(weights, "_version", -1))
        entry = _PARAM_CACHE.get(key)
        if entry is not None:
            ref, ver, cached = entry
            if ref() is weights and ver == version:
                return cached
        cached = _complex_to_interleaved(w.to(device))
        _PARAM_CACHE[key] = (weakref.ref(weights), version, cached)
        if len(_PARAM_CACHE) > _WEIGHT_CACHE_MAX * 2:
            for k in [k for k, (r, _, _) in _PARAM_CACHE.items() if r() is None]:
                _PARAM_CACHE.pop(k, None)
        return cached
    w_cpu = w.to("cpu", torch.complex64).resolve_conj().contiguous()
    digest = hashlib.blake2b(w_cpu.numpy().tobytes(), digest_size=16).hexdigest()
    key = (tuple(w_cpu.shape), digest, str(device))
    cached = _WEIGHT_DEVICE_CACHE.get(key)
    if cached is None:
        cached = _complex_to_interleaved(w_cpu.to(device))
        if len(_WEIGHT_DEVICE_CACHE) >= _WEIGHT_CACHE_MAX:
            _WEIGHT_DEVICE_CACHE.pop(next(iter(_WEIGHT_DEVICE_CACHE)))
        _WEIGHT_DEVICE_CACHE[key] = cached
    return cached


def clear_weight_supa_cache() -> None:
    """spectral_conv/spectral_conv_ops.py:191-196"""
    _WEIGHT_DEVICE_CACHE.clear()
    _PARAM_CACHE.clear()
    spectral_conv_ext._WORKSPACES.clear()


clear_weight_cache = clear_weight_supa_cache


def spectral_mul_supa(x_freq_modes: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """Single corner, complex in / CPU complex out (spectral_conv/spectral_conv_ops.py:127-138)."""
    device = _device_for(x_freq_modes)
    x_dev = _complex_to_interleaved(x_freq_modes.detach().to(device))
    w_dev = _weights_to_device_cached(weights, device)
    y = spectral_conv_ext.spectral_mul(x_dev, w_dev)
    return _interleaved_to_complex(y.cpu())


def spectral_mul_supa_device(x_freq_modes_interleaved: torch.Tensor, weights_interleaved: torch.Tensor,
                             synchronize: bool = False) -> torch.Tensor:
    """spectral_conv/spectral_conv_ops.py:141-152"""
    y = spectral_conv_ext.spectral_mul(x_freq_modes_interleaved.contiguous(), weights_interleaved.contiguous())
    if synchronize:
        torch.cuda.synchronize(y.device)
    return y


def spectral_mul_supa_out(x_freq_modes_interleaved: torch.Tensor, weights_interleaved: torch.Tensor,
                          out: torch.Tensor, synchronize: bool = False) -> torch.Tensor:
    """spectral_conv_combo/spectral_conv_ops.py:188-207"""
    spectral_conv_ext.spectral_mul_out(x_freq_modes_interleaved.contiguous(), weights_interleaved.contiguous(),
                                       out)
    if synchronize:
        torch.cuda.synchronize(out.device)
    return out


class SpectralMulFunction(torch.autograd.Function):
    """Device spectral_mul forward and backward (spectral_conv/spectral_conv_ops.py:260-278):
    the reference's two conjugate-transpose einsums run as the library's mixing kernel
    (scx_spectral_mul_bwd: per-mode conjugate transposes of w and x, then grad_y W^H and
    X^H grad_y), computing only the gradients autograd asks for."""

    @staticmethod
    def forward(ctx, x_freq_modes: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
        device = _device_for(x_freq_modes)
        x_c = x_freq_modes.detach().to(device, torch.complex64).resolve_conj().contiguous()
        w_c = weights.detach().to(device, torch.complex64).resolve_conj().contiguous()
        ctx.save_for_backward(x_c, w_c)
        ctx.out_device = x_freq_modes.device
        y = spectral_conv_ext.spectral_mul(torch.view_as_real(x_c), torch.view_as_real(w_c))
        return _interleaved_to_complex(y).to(x_freq_modes.device)

    @staticmethod
    def backward(ctx, grad_output: torch.Tensor):
        x_c, w_c = ctx.saved_tensors
        need_x, need_w = ctx.needs_input_grad[0], ctx.needs_input_grad[1]
        if not (need_x or need_w):
            return None, None
        grad_y = grad_output.to(x_c.device, torch.complex64).resolve_conj().contiguous()
        gx, gw = spectral_conv_ext.spectral_mul_backward(torch.view_as_real(x_c), torch.view_as_real(w_c),
                                                         torch.view_as_real(grad_y), need_x, need_w)
        grad_x = _interleaved_to_complex(gx).to(ctx.out_device) if need_x else None
        grad_w = _interleaved_to_complex(gw).to(ctx.out_device) if need_w else None
        return grad_x, grad_w


def spectral_mul_autograd(x_freq_modes: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """spectral_conv/spectral_conv_ops.py:281-286"""
    return SpectralMulFunction.apply(x_freq_modes, weights)


def resolve_use_sufft(height: int, width: int, use_sufft) -> bool:
    """Same rules and errors as spectral_conv/spectral_conv_ops.py:289-328.  Here the
    answer only selects the host-return contract of ``spectral_conv2d_v1``."""
    if isinstance(use_sufft, bool):
        return use_sufft
    if isinstance(use_sufft, str):
        key = use_sufft.strip().lower()
        if key in {"v1", "cpu"}:
            return False
        if key in {"fused", "sufft", "supa"}:
            return True
        if key in {"auto", "adaptive"}:
            cached = _AUTO_TUNE_TABLE.get(min(height, width))
            if cached is not None and "use_sufft" in cached:
                return bool(cached["use_sufft"])
            return min(height, width) >= 64
        raise ValueError(f"use_sufft string must be auto/v1/fused, got {use_sufft!r}")
    raise TypeError(f"use_sufft must be bool or str, got {type(use_sufft).__name__}")


def _to_device_input(x: torch.Tensor, device: torch.device) -> torch.Tensor:
    return x.detach().to(device=device, dtype=torch.float32).contiguous()


def spectral_conv2d_fused(x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                          modes2: int, *, to_cpu: bool = True, synchronize: bool | None = None) -> torch.Tensor:
    """Device-resident forward (spectral_conv/spectral_conv_ops.py:363-417): one truncated
    DFT kernel, one dual-corner mixing kernel, one inverse DFT kernel.  ``to_cpu=False``
    keeps the output on the device.  A page-locked float32 host input with a host result is
    streamed through in batch chunks by one native call (scx_spectral_conv2d_fwd_host)."""
    device = _device_for(x)
    w1 = _weights_to_device_cached(weights1, device)
    w2 = _weights_to_device_cached(weights2, device)
    if (to_cpu and not x.is_cuda and x.dim() == 4 and x.dtype == torch.float32 and x.is_contiguous()
            and x.is_pinned() and x.shape[0] > 1):
        return spectral_conv_ext.spectral_conv2d_fwd_host(x, w1, w2, int(modes1), int(modes2), device)
    x_dev = _to_device_input(x, device)
    y = spectral_conv_ext.spectral_conv2d_fwd(x_dev, w1, w2, int(modes1), int(modes2))
    if to_cpu:
        # a fresh page-locked tensor per call (torch's host caching allocator makes this
        # cheap), so the copy runs at full PCIe rate and results never alias
        host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        return host
    if synchronize:
        torch.cuda.current_stream(device).synchronize()
    return y


def spectral_conv2d_v1(x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                       modes2: int) -> torch.Tensor:
    """The reference's small-map path (spectral_conv/spectral_conv_ops.py:331-360) kept for
    its contract - it always returns a host tensor - but computed on the device."""
    return spectral_conv2d_fused(x, weights1, weights2, modes1, modes2, to_cpu=True)


def spectral_conv2d_supa(x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                         modes2: int, use_sufft="auto", *, to_cpu: bool = True,
                         synchronize: bool | None = None) -> torch.Tensor:
    """spectral_conv/spectral_conv_ops.py:480-505"""
    if x.dim() != 4:
        raise ValueError(f"x must be [B,C,H,W], got {tuple(x.shape)}")
    height, width = int(x.shape[-2]), int(x.shape[-1])
    if resolve_use_sufft(height, width, use_sufft):
        return spectral_conv2d_fused(x, weights1, weights2, modes1, modes2, to_cpu=to_cpu,
                                     synchronize=synchronize)
    return spectral_conv2d_v1(x, weights1, weights2, modes1, modes2)


def spectral_conv2d(x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                    modes2: int) -> torch.Tensor:
    """Neutral name: device in, device out (host input is moved to the current device)."""
    return spectral_conv2d_fused(x, weights1, weights2, modes1, modes2, to_cpu=False, synchronize=False)


def spectral_conv3d_supa(x: torch.Tensor, weights: torch.Tensor, modes1: int, modes2: int, modes3: int, *,
                         to_cpu: bool = True) -> torch.Tensor:
    """spectral_conv_combo/spectral_conv_ops.py:435-472, all on the device: the reference
    runs rfftn and irfftn on the CPU around a device mixing; here the truncated DFTs, the
    mixing and the inverse are one library call.  Returns a host tensor like the reference
    (``to_cpu=False`` keeps it on the device)."""
    if x.dim() != 5:
        raise ValueError(f"x must be [B,C,D,H,W], got {tuple(x.shape)}")
    device = _device_for(x)
    x_dev = x.detach().to(device=device, dtype=torch.float32).contiguous()
    w = weights.detach()
    w_dev = w.to(device=device, dtype=torch.complex64) if w.is_complex() else w.to(device=device)
    y = spectral_conv_ext.spectral_conv3d_fwd(x_dev, w_dev, int(modes1), int(modes2), int(modes3))
    if to_cpu:
        host = torch.empty(y.shape, dtype=y.dtype, pin_memory=True)
        host.copy_(y, non_blocking=True)
        torch.cuda.current_stream(device).synchronize()
        return host
    return y


class SpectralConv3d(nn.Module):
    """The four-corner 3-D layer of spectral_conv_combo/official_baseline.py:60-100: same
    parameters (weights1..4 = scale * rand(cfloat), scale = 1/(Cin Cout)) and construction
    order, so state dicts load; forward runs on the module's device and returns a device
    tensor (scx_spectral_conv3d_4c_fwd)."""

    def __init__(self, in_channels: int, out_channels: int, modes1: int, modes2: int, modes3: int):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.modes1 = modes1
        self.modes2 = modes2
        self.modes3 = modes3
        scale = 1.0 / (in_channels * out_channels)
        shape = (in_channels, out_channels, modes1, modes2, modes3)
        self.weights1 = nn.Parameter(scale * torch.rand(*shape, dtype=torch.cfloat))
        self.weights2 = nn.Parameter(scale * torch.rand(*shape, dtype=torch.cfloat))
        self.weights3 = nn.Parameter(scale * torch.rand(*shape, dtype=torch.cfloat))
        self.weights4 = nn.Parameter(scale * torch.rand(*shape, dtype=torch.cfloat))

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        device = self.weights1.device
        if device.type != "cuda":
            raise RuntimeError("SpectralConv3d runs on a CUDA device: move the module with .cuda()")
        x_dev = x.detach().to(device=device, dtype=torch.float32).contiguous()
        ws = [w.detach() for w in (self.weights1, self.weights2, self.weights3, self.weights4)]
        return spectral_conv_ext.spectral_conv3d_4c_fwd(x_dev, ws, self.modes1, self.modes2, self.modes3)


def warmup_spectral_plans(height: int = 256, width: int = 256, channels_in: int = 32, channels_out: int = 64,
                          modes1: int = 16, modes2: int = 16, batch_size: int = 4) -> None:
    """Builds the shape's twiddle tables and runs the fused path once, outside any stream
    capture (spectral_conv/spectral_conv_ops.py:459-477)."""
    device = _device_for(torch.empty(0))
    with torch.cuda.device(device):
        spectral_conv_ext.prepare(height, width, modes1, modes2)
    x = torch.randn(batch_size, channels_in, height, width, dtype=torch.float32, device=device)
    scale = 1.0 / (channels_in * channels_out)
    w1 = scale * torch.rand(channels_in, channels_out, modes1, modes2, dtype=torch.cfloat, device=device)
    w2 = scale * torch.rand(channels_in, channels_out, modes1, modes2, dtype=torch.cfloat, device=device)
    spectral_conv2d_fused(x, w1, w2, modes1, modes2, to_cpu=False)
    torch.cuda.synchronize(device)


class SpectralConv2dSupa(nn.Module):
    """spectral_conv/spectral_conv_ops.py:508-536: same parameters and init."""

    def __init__(self, in_channels: int, out_channels: int, modes1: int, modes2: int):
        super().__init__()
        self.modes1 = modes1
        self.modes2 = modes2
        scale = 1.0 / (in_channels * out_channels)
        self.weights1 = nn.Parameter(scale * torch.rand(in_channels, out_channels, modes1, modes2,
                                                        dtype=torch.cfloat))
        self.weights2 = nn.Parameter(scale * torch.rand(in_channels, out_channels, modes1, modes2,
                                                        dtype=torch.cfloat))

    def forward(self, x: torch.Tensor, use_sufft="auto", *, to_cpu: bool = True) -> torch.Tensor:
        return spectral_conv2d_supa(x, self.weights1, self.weights2, self.modes1, self.modes2,
                                    use_sufft=use_sufft, to_cpu=to_cpu)


class SpectralConv2dFunction(torch.autograd.Function):
    """Differentiable SpectralConv2d on the device: the fused forward keeps the input corner
    spectra, and the backward (scx_spectral_conv2d_bwd) returns the gradients torch autograd
    gives for spectral_conv/reference_pytorch.py:30-47.  The reference differentiates only
    the mixing (SpectralMulFunction, spectral_conv/spectral_conv_ops.py:260-286)."""

    @staticmethod
    def forward(ctx, x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                modes2: int) -> torch.Tensor:
        device = x.device
        w1 = _weights_to_device_cached(weights1, device)
        w2 = _weights_to_device_cached(weights2, device)
        y, x_corners = spectral_conv_ext.spectral_conv2d_fwd_saved(
            x.detach().to(torch.float32).contiguous(), w1, w2, int(modes1), int(modes2))
        ctx.x_corners = x_corners
        ctx.w = (w1, w2)
        ctx.modes = (int(modes1), int(modes2))
        ctx.x_dtype = x.dtype
        ctx.w_complex = (weights1.is_complex(), weights2.is_complex())
        return y

    @staticmethod
    def backward(ctx, grad_y: torch.Tensor):
        need_x, need_w1, need_w2 = ctx.needs_input_grad[:3]
        gx, gw1, gw2 = spectral_conv_ext.spectral_conv2d_bwd(
            grad_y.to(torch.float32), ctx.x_corners, ctx.w[0], ctx.w[1], *ctx.modes, need_x=need_x,
            need_w=need_w1 or need_w2)
        if gx is not None:
            gx = gx.to(ctx.x_dtype)
        if gw1 is not None:
            gw1 = torch.view_as_complex(gw1) if ctx.w_complex[0] else gw1
            gw2 = torch.view_as_complex(gw2) if ctx.w_complex[1] else gw2
        ctx.x_corners = None
        return gx, (gw1 if need_w1 else None), (gw2 if need_w2 else None), None, None


def spectral_conv2d_autograd(x: torch.Tensor, weights1: torch.Tensor, weights2: torch.Tensor, modes1: int,
                             modes2: int) -> torch.Tensor:
    """Device-resident SpectralConv2d forward that autograd can differentiate (x a CUDA
    tensor; weights complex64 [Cin,Cout,m1,m2] or interleaved float32 on its device)."""
    if not x.is_cuda:
        raise RuntimeError("spectral_conv2d_autograd needs a CUDA input")
    return SpectralConv2dFunction.apply(x, weights1, weights2, modes1, modes2)


class SpectralConv2d(nn.Module):
    """State-dict compatible with spectral_conv/reference_pytorch.py:12-25; forward runs on
    the module's device (move it with ``.cuda()``) and returns a device tensor."""

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

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if torch.is_grad_enabled() and x.is_cuda and (x.requires_grad or self.weights1.requires_grad
                                                       or self.weights2.requires_grad):
            return spectral_conv2d_autograd(x, self.weights1, self.weights2, self.modes1, self.modes2)
        return spectral_conv2d(x, self.weights1, self.weights2, self.modes1, self.modes2)
