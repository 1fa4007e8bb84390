"""Drop-in for the reference's native module ``spectral_conv_ext``
(spectral_conv/spectral_conv_ext.cpp:386-409), backed by libscx.so on a CUDA device.

Same function names, argument meaning and checks; a failed check raises RuntimeError the
way TORCH_CHECK does.  Differences that fix reference defects:
* kernels run on the current CUDA stream, not the null stream (spectral_conv_ext.cpp:148);
* ``spectral_mul_dual_scatter_out`` writes the corners into rows [0, m1) and [H-m1, H) of
  ``out_freq`` itself (the reference narrows dim 2 at ``Wf-M1`` and writes into a
  contiguous copy, so its writes never land: spectral_conv_ext.cpp:286-289).
New: ``spectral_conv2d_fwd`` runs the whole fused forward in one call.
"""

from __future__ import annotations

import torch

import _scx


def _check(cond: bool, *msg) -> None:
    if not cond:
        raise RuntimeError("".join(str(m) for m in msg))


def _check_freq_tensor(t: torch.Tensor, name: str) -> None:
    """spectral_conv/spectral_conv_ext.cpp:26-31"""
    _check(t.dim() == 5, name, " must have shape [..., 2] interleaved complex")
    _check(t.size(-1) == 2, name, " last dim must be 2 (real,imag)")
    _check(t.dtype == torch.float32, name, " must be float32")
    _check(t.is_contiguous(), name, " must be contiguous")
    _check(t.is_cuda, name, " must be a CUDA tensor")


def spectral_mul(x_freq: torch.Tensor, weights: torch.Tensor) -> torch.Tensor:
    """y[b,o,k] = sum_i x[b,i,k] w[i,o,k]; spectral_conv/spectral_conv_ext.cpp:123-151."""
    _check_freq_tensor(x_freq, "x_freq")
    _check_freq_tensor(weights, "weights")
    _check(x_freq.device == weights.device, "x_freq and weights must share device")
    B, Cin, m1, m2 = (int(s) for s in x_freq.shape[:4])
    Cout = int(weights.size(1))
    _check(weights.size(0) == Cin, "weights C_in mismatch")
    _check(weights.size(2) == m1 and weights.size(3) == m2, "modes mismatch")
    _check(B > 0 and Cin > 0 and Cout > 0 and m1 > 0 and m2 > 0, "sizes must be positive")
    y = torch.empty(B, Cout, m1, m2, 2, device=x_freq.device, dtype=torch.float32)
    with _scx.device_guard(x_freq.device):
        _scx.check(_scx.lib.scx_spectral_mul(x_freq.data_ptr(), weights.data_ptr(), y.data_ptr(), B, Cin,
                                             Cout, m1, m2, _scx.stream_of(x_freq.device)),
                   "launch_spectral_mul")
    return y


def spectral_mul_out(x_freq: torch.Tensor, weights: torch.Tensor, y_freq: torch.Tensor) -> None:
    """In-place variant into ``y_freq``; spectral_conv/spectral_conv_ext.cpp:164-193."""
    _check_freq_tensor(x_freq, "x_freq")
    _check_freq_tensor(weights, "weights")
    _check_freq_tensor(y_freq, "y_freq")
    _check(x_freq.device == weights.device, "x_freq and weights must share device")
    _check(x_freq.device == y_freq.device, "y_freq must share device with x_freq")
    B, Cin, m1, m2 = (int(s) for s in x_freq.shape[:4])
    Cout = int(weights.size(1))
    _check(y_freq.size(0) == B, "y_freq batch mismatch")
    _check(y_freq.size(1) == Cout, "y_freq C_out mismatch")
    _check(y_freq.size(2) == m1 and y_freq.size(3) == m2, "y_freq modes mismatch")
    _check(weights.size(0) == Cin, "weights C_in mismatch")
    _check(weights.size(2) == m1 and weights.size(3) == m2, "weights modes mismatch")
    with _scx.device_guard(x_freq.device):
        _scx.check(_scx.lib.scx_spectral_mul(x_freq.data_ptr(), weights.data_ptr(), y_freq.data_ptr(), B,
                                             Cin, Cout, m1, m2, _scx.stream_of(x_freq.device)),
                   "launch_spectral_mul(out)")


def spectral_mul_backward(x_freq: torch.Tensor | None, weights: torch.Tensor | None, grad_y: torch.Tensor,
                          need_x: bool = True, need_w: bool = True):
    """Gradients of ``spectral_mul`` (the backward of SpectralMulFunction,
    spectral_conv/spectral_conv_ops.py:272-278) on the device: grad_x = grad_y W^H and
    grad_w = X^H grad_y per mode.  Interleaved [...,2] float32 tensors as for spectral_mul;
    returns (grad_x or None, grad_w or None)."""
    _check_freq_tensor(grad_y, "grad_y")
    _check(need_x or need_w, "nothing to compute")
    B, Cout, m1, m2 = (int(s) for s in grad_y.shape[:4])
    if need_x:
        _check_freq_tensor(weights, "weights")
        Cin = int(weights.size(0))
        _check(weights.size(1) == Cout and weights.size(2) == m1 and weights.size(3) == m2, "weights shape mismatch")
    if need_w:
        _check_freq_tensor(x_freq, "x_freq")
        Cin = int(x_freq.size(1))
        _check(x_freq.size(0) == B and x_freq.size(2) == m1 and x_freq.size(3) == m2, "x_freq shape mismatch")
    dev = grad_y.device
    gx = torch.empty(B, Cin, m1, m2, 2, device=dev) if need_x else None
    gw = torch.empty(Cin, Cout, m1, m2, 2, device=dev) if need_w else None
    nbytes = _scx.lib.scx_spectral_mul_bwd_workspace_size(B, Cin, Cout, m1, m2)
    _check(nbytes > 0, "invalid sizes")
    with _scx.device_guard(dev):
        ws = torch.empty(nbytes, dtype=torch.uint8, device=dev)
        _scx.check(_scx.lib.scx_spectral_mul_bwd(x_freq.data_ptr() if need_w else None,
                                                 weights.data_ptr() if need_x else None, grad_y.data_ptr(),
                                                 gx.data_ptr() if need_x else None, gw.data_ptr() if need_w else None,
                                                 B, Cin, Cout, m1, m2, ws.data_ptr(), nbytes, _scx.stream_of(dev)),
                   "scx_spectral_mul_bwd")
    return gx, gw


def _check_dual(x1, w1, y1, x2, w2, y2) -> tuple[int, int, int, int, int]:
    def one(xn, wn, yn, prefix):
        _check_freq_tensor(xn, prefix)
        _check_freq_tensor(wn, "weights")
        _check_freq_tensor(yn, "y_freq")
        _check(xn.device == wn.device, "x and weights must share device")
        _check(xn.device == yn.device, "y must share device with x")
        _check(xn.size(0) == yn.size(0), "y batch mismatch")
        _check(xn.size(1) == wn.size(0), "weights C_in mismatch")
        _check(yn.size(1) == wn.size(1), "y C_out mismatch")
        _check(xn.size(2) == wn.size(2) and xn.size(2) == yn.size(2), "modes1 mismatch")
        _check(xn.size(3) == wn.size(3) and xn.size(3) == yn.size(3), "modes2 mismatch")

    one(x1, w1, y1, "x_freq1")
    one(x2, w2, y2, "x_freq2")
    _check(x1.shape == x2.shape and w1.shape == w2.shape and y1.shape == y2.shape,
           "corner shapes must match")
    _check(x1.device == x2.device, "x1 and x2 must share device")
    return int(x1.size(0)), int(x1.size(1)), int(w1.size(1)), int(x1.size(2)), int(x1.size(3))


def spectral_mul_dual_out(x1, w1, x2, w2, y1, y2) -> None:
    """Both corners in ONE launch; spectral_conv/spectral_conv_ext.cpp:200-245."""
    B, Cin, Cout, m1, m2 = _check_dual(x1, w1, y1, x2, w2, y2)
    with _scx.device_guard(x1.device):
        _scx.check(_scx.lib.scx_spectral_mul_dual(x1.data_ptr(), x2.data_ptr(), w1.data_ptr(), w2.data_ptr(),
                                                  y1.data_ptr(), y2.data_ptr(), B, Cin, Cout, m1, m2,
                                                  _scx.stream_of(x1.device)),
                   "launch_spectral_mul(dual)")


def spectral_mul_dual_scatter_out(x1, w1, x2, w2, out_freq) -> None:
    """Zeroes ``out_freq`` [B,Cout,H,Wf,2] and writes the two mixed corners into rows
    [0, m1) and [H-m1, H), columns [0, m2): the intent of
    spectral_conv/spectral_conv_ext.cpp:257-311 (whose writes never land)."""
    _check_freq_tensor(out_freq, "out_freq")
    B, Cin, m1, m2 = (int(s) for s in x1.shape[:4])
    Cout = int(w1.size(1))
    _check(out_freq.size(0) == B and out_freq.size(1) == Cout, "out_freq batch/C_out mismatch")
    _check(m2 <= out_freq.size(3), "modes2 must fit within width_freq")
    _check(m1 <= out_freq.size(2), "modes1 must fit within height")
    y1 = torch.empty(B, Cout, m1, m2, 2, device=out_freq.device, dtype=torch.float32)
    y2 = torch.empty_like(y1)
    spectral_mul_dual_out(x1, w1, x2, w2, y1, y2)
    out_freq.zero_()
    H = out_freq.size(2)
    out_freq[:, :, :m1, :m2] = y1
    out_freq[:, :, H - m1:, :m2] = y2


def rfft2_sufft(x: torch.Tensor) -> torch.Tensor:
    """Full half-spectrum [B,C,H,W//2+1,2]; spectral_conv/spectral_conv_ext.cpp:314-347."""
    _check(x.dim() == 4, "rfft2_sufft expects [B,C,H,W]")
    _check(x.dtype == torch.float32, "rfft2_sufft expects float32")
    _check(x.is_cuda, "rfft2_sufft expects a CUDA tensor")
    x = x.contiguous()
    B, C, H, W = (int(s) for s in x.shape)
    out = torch.empty(B, C, H, W // 2 + 1, 2, device=x.device, dtype=torch.float32)
    with _scx.device_guard(x.device):
        _scx.check(_scx.lib.scx_rfft2(x.data_ptr(), out.data_ptr(), B, C, H, W, _scx.stream_of(x.device)),
                   "rfft2")
    return out


def irfft2_sufft(x_freq: torch.Tensor, height: int, width: int) -> torch.Tensor:
    """[B,C,H,W//2+1,2] -> [B,C,H,W] with 1/(HW); spectral_conv/spectral_conv_ext.cpp:349-384."""
    _check_freq_tensor(x_freq, "x_freq")
    B, C = int(x_freq.size(0)), int(x_freq.size(1))
    _check(x_freq.size(2) == height, "height mismatch")
    _check(x_freq.size(3) == width // 2 + 1, "width_freq mismatch")
    out = torch.empty(B, C, height, width, device=x_freq.device, dtype=torch.float32)
    with _scx.device_guard(x_freq.device):
        _scx.check(_scx.lib.scx_irfft2(x_freq.data_ptr(), out.data_ptr(), B, C, int(height), int(width),
                                       _scx.stream_of(x_freq.device)), "irfft2")
    return out


def rfft2_corners(x: torch.Tensor, modes1: int, modes2: int):
    """Truncated forward DFT: x [B,C,H,W] -> (corner1, corner2) [B,C,m1,m2,2]."""
    _check(x.dim() == 4 and x.dtype == torch.float32 and x.is_cuda, "x must be float32 CUDA [B,C,H,W]")
    x = x.contiguous()
    B, C, H, W = (int(s) for s in x.shape)
    x1 = torch.empty(B, C, modes1, modes2, 2, device=x.device, dtype=torch.float32)
    x2 = torch.empty_like(x1)
    with _scx.device_guard(x.device):
        _scx.check(_scx.lib.scx_rfft2_corners(x.data_ptr(), x1.data_ptr(), x2.data_ptr(), B, C, H, W,
                                              int(modes1), int(modes2), _scx.stream_of(x.device)),
                   "rfft2_corners")
    return x1, x2


def irfft2_corners(y1: torch.Tensor, y2: torch.Tensor, height: int, width: int) -> torch.Tensor:
    """Zero-padded inverse from the two corners [B,C,m1,m2,2] -> y [B,C,H,W]."""
    _check_freq_tensor(y1, "y1")
    _check_freq_tensor(y2, "y2")
    _check(y1.shape == y2.shape and y1.device == y2.device, "corner shapes/devices must match")
    B, C, m1, m2 = (int(s) for s in y1.shape[:4])
    y = torch.empty(B, C, height, width, device=y1.device, dtype=torch.float32)
    with _scx.device_guard(y1.device):
        _scx.check(_scx.lib.scx_irfft2_corners(y1.data_ptr(), y2.data_ptr(), y.data_ptr(), B, C, int(height),
                                               int(width), m1, m2, _scx.stream_of(y1.device)),
                   "irfft2_corners")
    return y


_WORKSPACES: dict = {}


def workspace(nbytes: int, device: torch.device) -> torch.Tensor:
    """Grow-only scratch for the fused forward (the two corner spectra), one per
    (device, current stream) so that calls on different streams never share it."""
    key = (device.type, device.index, _scx.stream_of(device))
    buf = _WORKSPACES.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _WORKSPACES[key] = buf
    return buf


def spectral_conv2d_fwd(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, modes1: int, modes2: int,
                        out: torch.Tensor | None = None) -> torch.Tensor:
    """Fused SpectralConv2d forward on the device.  x [B,Cin,H,W] float32 CUDA; w1/w2
    [Cin,Cout,m1,m2,2] float32 (interleaved) or complex64 on the same device."""
    _check(x.dim() == 4, "x must be [B,C,H,W]")
    _check(x.is_cuda and x.dtype == torch.float32 and x.is_contiguous(), "x must be contiguous float32 CUDA")
    if w1.is_complex():
        w1 = torch.view_as_real(w1.resolve_conj().contiguous())
    if w2.is_complex():
        w2 = torch.view_as_real(w2.resolve_conj().contiguous())
    _check_freq_tensor(w1, "weights1")
    _check_freq_tensor(w2, "weights2")
    _check(w1.shape == w2.shape, "weights1/weights2 shape mismatch")
    _check(w1.device == x.device and w2.device == x.device, "weights must be on x.device")
    B, Cin, H, W = (int(s) for s in x.shape)
    _check(w1.size(0) == Cin, "weights C_in mismatch")
    _check(w1.size(2) == modes1 and w1.size(3) == modes2, "weights modes mismatch")
    Cout = int(w1.size(1))
    _check(1 <= modes1 <= H and 1 <= modes2 <= W // 2 + 1, "modes out of range for the grid")
    if out is None:
        out = torch.empty(B, Cout, H, W, device=x.device, dtype=torch.float32)
    else:
        _check(out.shape == (B, Cout, H, W) and out.is_contiguous() and out.dtype == torch.float32
               and out.device == x.device, "out must be a contiguous float32 [B,Cout,H,W] on x.device")
    lib = _scx.lib
    need = lib.scx_spectral_conv2d_workspace_size(B, Cin, Cout, H, W, int(modes1), int(modes2))
    _check(need > 0, "invalid SpectralConv2d sizes")
    ws = workspace(need, x.device)
    with _scx.device_guard(x.device):
        _scx.check(lib.scx_spectral_conv2d_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), out.data_ptr(), B,
                                               Cin, Cout, H, W, int(modes1), int(modes2), ws.data_ptr(),
                                               ws.numel(), _scx.stream_of(x.device)),
                   "spectral_conv2d_fwd")
    return out


def spectral_conv2d_fwd_host(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, modes1: int, modes2: int,
                             device: torch.device, out: torch.Tensor | None = None, chunks: int = 0) -> torch.Tensor:
    """Fused SpectralConv2d forward from a host tensor to a host tensor through
    scx_spectral_conv2d_fwd_host: the batch is streamed through the device in chunks whose
    uploads, forwards and downloads overlap.  x [B,Cin,H,W] contiguous float32 on the CPU
    (page-locked for the overlap); w1/w2 as for spectral_conv2d_fwd, on ``device``.  Returns
    a page-locked [B,Cout,H,W] host tensor (or fills ``out``) once the result is there."""
    _check(x.dim() == 4, "x must be [B,C,H,W]")
    _check(not x.is_cuda and x.dtype == torch.float32 and x.is_contiguous(),
           "x must be a contiguous float32 host tensor")
    if w1.is_complex():
        w1 = torch.view_as_real(w1.resolve_conj().contiguous())
    if w2.is_complex():
        w2 = torch.view_as_real(w2.resolve_conj().contiguous())
    _check_freq_tensor(w1, "weights1")
    _check_freq_tensor(w2, "weights2")
    _check(w1.shape == w2.shape, "weights1/weights2 shape mismatch")
    _check(w1.device == device and w2.device == device, "weights must be on the device")
    B, Cin, H, W = (int(s) for s in x.shape)
    _check(w1.size(0) == Cin, "weights C_in mismatch")
    _check(w1.size(2) == modes1 and w1.size(3) == modes2, "weights modes mismatch")
    Cout = int(w1.size(1))
    _check(1 <= modes1 <= H and 1 <= modes2 <= W // 2 + 1, "modes out of range for the grid")
    if out is None:
        out = torch.empty(B, Cout, H, W, dtype=torch.float32, pin_memory=True)
    else:
        _check(out.shape == (B, Cout, H, W) and out.is_contiguous() and out.dtype == torch.float32
               and not out.is_cuda, "out must be a contiguous float32 [B,Cout,H,W] host tensor")
    lib = _scx.lib
    need = lib.scx_spectral_conv2d_workspace_size(B, Cin, Cout, H, W, int(modes1), int(modes2))
    _check(need > 0, "invalid SpectralConv2d sizes")
    ws = workspace(need, device)
    x_dev = torch.empty(B, Cin, H, W, dtype=torch.float32, device=device)
    y_dev = torch.empty(B, Cout, H, W, dtype=torch.float32, device=device)
    with _scx.device_guard(device):
        _scx.check(lib.scx_spectral_conv2d_fwd_host(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), out.data_ptr(), B,
                                                    Cin, Cout, H, W, int(modes1), int(modes2), x_dev.data_ptr(),
                                                    y_dev.data_ptr(), ws.data_ptr(), ws.numel(), int(chunks),
                                                    _scx.stream_of(device)),
                   "spectral_conv2d_fwd_host")
    return out


def spectral_conv2d_fwd_saved(x: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, modes1: int,
                              modes2: int) -> tuple:
    """spectral_conv2d_fwd that also keeps the input corner spectra for the backward:
    returns (y, x_corners), x_corners [2,B,Cin,m1,m2,2] float32 (corner 1, corner 2) - the
    head of a workspace of its own, where the forward leaves them."""
    _check(x.dim() == 4 and x.is_cuda and x.dtype == torch.float32 and x.is_contiguous(),
           "x must be contiguous float32 CUDA [B,C,H,W]")
    w1 = torch.view_as_real(w1.resolve_conj().contiguous()) if w1.is_complex() else w1
    w2 = torch.view_as_real(w2.resolve_conj().contiguous()) if w2.is_complex() else w2
    _check_freq_tensor(w1, "weights1")
    _check_freq_tensor(w2, "weights2")
    _check(w1.shape == w2.shape and w1.device == x.device and w2.device == x.device,
           "weights must match and be on x.device")
    B, Cin, H, W = (int(s) for s in x.shape)
    _check(w1.size(0) == Cin and w1.size(2) == modes1 and w1.size(3) == modes2, "weights shape mismatch")
    _check(1 <= modes1 <= H and 1 <= modes2 <= W // 2 + 1, "modes out of range for the grid")
    Cout = int(w1.size(1))
    lib = _scx.lib
    need = lib.scx_spectral_conv2d_workspace_size(B, Cin, Cout, H, W, int(modes1), int(modes2))
    _check(need > 0, "invalid SpectralConv2d sizes")
    ws = torch.empty(need, dtype=torch.uint8, device=x.device)
    y = torch.empty(B, Cout, H, W, device=x.device, dtype=torch.float32)
    with _scx.device_guard(x.device):
        _scx.check(lib.scx_spectral_conv2d_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), B, Cin,
                                               Cout, H, W, int(modes1), int(modes2), ws.data_ptr(), ws.numel(),
                                               _scx.stream_of(x.device)),
                   "spectral_conv2d_fwd")
    n = 2 * B * Cin * modes1 * modes2 * 2
    x_corners = ws[: n * 4].view(torch.float32).view(2, B, Cin, modes1, modes2, 2)
    return y, x_corners


def spectral_conv2d_bwd(grad_y: torch.Tensor, x_corners: torch.Tensor | None, w1: torch.Tensor, w2: torch.Tensor,
                        modes1: int, modes2: int, need_x: bool = True, need_w: bool = True) -> tuple:
    """SpectralConv2d backward through scx_spectral_conv2d_bwd: (grad_x or None, grad_w1 or
    None, grad_w2 or None), weight gradients as interleaved [Cin,Cout,m1,m2,2] float32.
    x_corners is the second result of spectral_conv2d_fwd_saved (needed for weight grads)."""
    _check(grad_y.dim() == 4 and grad_y.is_cuda and grad_y.dtype == torch.float32,
           "grad_y must be float32 CUDA [B,Cout,H,W]")
    grad_y = grad_y.contiguous()
    w1 = torch.view_as_real(w1.resolve_conj().contiguous()) if w1.is_complex() else w1.contiguous()
    w2 = torch.view_as_real(w2.resolve_conj().contiguous()) if w2.is_complex() else w2.contiguous()
    _check_freq_tensor(w1, "weights1")
    _check(w1.shape == w2.shape, "weights1/weights2 shape mismatch")
    B, Cout, H, W = (int(s) for s in grad_y.shape)
    Cin = int(w1.size(0))
    _check(int(w1.size(1)) == Cout and w1.size(2) == modes1 and w1.size(3) == modes2, "weights shape mismatch")
    dev = grad_y.device
    grad_x = torch.empty(B, Cin, H, W, device=dev, dtype=torch.float32) if need_x else None
    gw1 = torch.empty_like(w1) if need_w else None
    gw2 = torch.empty_like(w2) if need_w else None
    if need_w:
        _check(x_corners is not None and x_corners.is_contiguous()
               and tuple(x_corners.shape) == (2, B, Cin, modes1, modes2, 2), "x_corners shape mismatch")
    lib = _scx.lib
    need = lib.scx_spectral_conv2d_bwd_workspace_size(B, Cin, Cout, H, W, int(modes1), int(modes2))
    _check(need > 0, "invalid SpectralConv2d sizes")
    ws = torch.empty(need, dtype=torch.uint8, device=dev)
    ptr = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    with _scx.device_guard(dev):
        _scx.check(lib.scx_spectral_conv2d_bwd(grad_y.data_ptr(), ptr(x_corners) if need_w else None,
                                               w1.data_ptr(), w2.data_ptr(), ptr(grad_x), ptr(gw1), ptr(gw2), B, Cin,
                                               Cout, H, W, int(modes1), int(modes2), ws.data_ptr(), ws.numel(),
                                               _scx.stream_of(dev)),
                   "spectral_conv2d_bwd")
    return grad_x, gw1, gw2


def spectral_conv3d_fwd(x: torch.Tensor, w: torch.Tensor, modes1: int, modes2: int, modes3: int) -> torch.Tensor:
    """Single-corner SpectralConv3d forward on the device (scx_spectral_conv3d_fwd): x
    [B,Cin,D,H,W] float32 CUDA; w [Cin,Cout,m1,m2,m3] complex64 (or [...,2] float32) on the
    same device; returns y [B,Cout,D,H,W]."""
    _check(x.dim() == 5 and x.is_cuda and x.dtype == torch.float32, "x must be float32 CUDA [B,C,D,H,W]")
    x = x.contiguous()
    if w.is_complex():
        w = torch.view_as_real(w.to(torch.complex64).resolve_conj().contiguous())
    _check(w.dim() == 6 and w.size(-1) == 2 and w.dtype == torch.float32 and w.is_contiguous(),
           "weights must be [C_in,C_out,m1,m2,m3] complex64 or [...,2] float32")
    _check(w.device == x.device, "weights must be on x.device")
    B, Cin, D, H, W = (int(s) for s in x.shape)
    _check(int(w.size(0)) == Cin and tuple(int(v) for v in w.shape[2:5]) == (modes1, modes2, modes3),
           "weights shape mismatch")
    Cout = int(w.size(1))
    lib = _scx.lib
    need = lib.scx_spectral_conv3d_workspace_size(B, Cin, Cout, D, H, W, int(modes1), int(modes2), int(modes3))
    _check(need > 0, "invalid SpectralConv3d sizes (m1 <= D, m2 <= H, m3 <= W/2+1)")
    ws = workspace(need, x.device)
    y = torch.empty(B, Cout, D, H, W, device=x.device, dtype=torch.float32)
    with _scx.device_guard(x.device):
        _scx.check(lib.scx_spectral_conv3d_fwd(x.data_ptr(), w.data_ptr(), y.data_ptr(), B, Cin, Cout, D, H, W,
                                               int(modes1), int(modes2), int(modes3), ws.data_ptr(), ws.numel(),
                                               _scx.stream_of(x.device)),
                   "spectral_conv3d_fwd")
    return y


def spectral_conv3d_4c_fwd(x: torch.Tensor, ws: list, modes1: int, modes2: int, modes3: int) -> torch.Tensor:
    """Four-corner SpectralConv3d forward on the device (scx_spectral_conv3d_4c_fwd): ws =
    [w1, w2, w3, w4], each [Cin,Cout,m1,m2,m3] complex64 (or [...,2] float32) on x's device."""
    _check(x.dim() == 5 and x.is_cuda and x.dtype == torch.float32, "x must be float32 CUDA [B,C,D,H,W]")
    _check(len(ws) == 4, "four corner weights")
    x = x.contiguous()
    wr = []
    for w in ws:
        if w.is_complex():
            w = torch.view_as_real(w.to(torch.complex64).resolve_conj().contiguous())
        _check(w.dim() == 6 and w.size(-1) == 2 and w.dtype == torch.float32 and w.is_contiguous()
               and w.device == x.device, "weights must be [C_in,C_out,m1,m2,m3] complex on x.device")
        wr.append(w)
    B, Cin, D, H, W = (int(s) for s in x.shape)
    for w in wr:
        _check(w.shape == wr[0].shape and int(w.size(0)) == Cin
               and tuple(int(v) for v in w.shape[2:5]) == (modes1, modes2, modes3), "weights shape mismatch")
    Cout = int(wr[0].size(1))
    lib = _scx.lib
    need = lib.scx_spectral_conv3d_4c_workspace_size(B, Cin, Cout, D, H, W, int(modes1), int(modes2), int(modes3))
    _check(need > 0, "invalid SpectralConv3d sizes (m1 <= D, m2 <= H, m3 <= W/2+1)")
    wsb = workspace(need, x.device)
    y = torch.empty(B, Cout, D, H, W, device=x.device, dtype=torch.float32)
    with _scx.device_guard(x.device):
        _scx.check(lib.scx_spectral_conv3d_4c_fwd(x.data_ptr(), wr[0].data_ptr(), wr[1].data_ptr(), wr[2].data_ptr(),
                                                  wr[3].data_ptr(), y.data_ptr(), B, Cin, Cout, D, H, W, int(modes1),
                                                  int(modes2), int(modes3), wsb.data_ptr(), wsb.numel(),
                                                  _scx.stream_of(x.device)),
                   "spectral_conv3d_4c_fwd")
    return y


def prepare(height: int, width: int, modes1: int, modes2: int) -> None:
    """Builds the twiddle tables of one shape on the current device (outside capture)."""
    _scx.check(_scx.lib.scx_prepare(int(height), int(width), int(modes1), int(modes2)), "prepare")
