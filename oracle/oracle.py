"""ORACLE - TEST INFRASTRUCTURE ONLY.

CPU restatements of the reference's SpectralConv2d / FNO-2d forward, used only by
``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg as the checker.
The product path (``spectral_conv_ops`` -> ``libscx.so``) never imports this module.

Three independent restatements of ``spectral_conv/reference_pytorch.py:30-47``:

* ``spectral_conv2d_f64``   - direct DFTs in float64 C (``scx_oracle.c``), no FFT library;
* ``spectral_conv2d_np``    - numpy float64 FFT (pocketfft in numpy);
* ``spectral_conv2d_torch`` - the reference's own torch.fft / einsum recipe on the CPU in
  fp32 (the path the reference times as its CPU baseline).

and of the FNO forward ``fno_ns/model.py:183-198`` (``FNO2d.forward(use_supa=False)``):
``fno2d_torch``; and of the single-corner SpectralConv3d
(``spectral_conv_combo/reference_pytorch.py:51-82``): ``spectral_conv3d_np``.
``spectral_conv2d_grads_torch`` differentiates the torch recipe (float64
autograd) for the SpectralConv2d backward.  All are pinned against fixtures produced by the reference itself
(``tests/golden/make_golden.py``).
"""

from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "libscx_oracle.so"
_lib = None


def build() -> Path:
    """Compiles the float64 C restatement (``make -C oracle``)."""
    subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is None:
        if not _LIB_PATH.exists():
            build()
        lib = ctypes.CDLL(str(_LIB_PATH))
        f64p = ctypes.POINTER(ctypes.c_double)
        f32p = ctypes.POINTER(ctypes.c_float)
        lib.oracle_spectral_conv2d.argtypes = [f32p, f32p, f32p, f64p] + [ctypes.c_int] * 7
        lib.oracle_spectral_conv2d.restype = ctypes.c_int
        lib.oracle_rfft2_corners.argtypes = [f32p, f64p, f64p] + [ctypes.c_int] * 5
        lib.oracle_rfft2_corners.restype = ctypes.c_int
        _lib = lib
    return _lib


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _interleaved(w) -> np.ndarray:
    """complex [Cin,Cout,m1,m2] (or already [...,2] float) -> float32 [...,2]."""
    w = np.asarray(w)
    if np.iscomplexobj(w):
        w = np.stack([w.real, w.imag], axis=-1)
    return _f32(w)


def _ptr(a: np.ndarray, ctype):
    return a.ctypes.data_as(ctypes.POINTER(ctype))


def spectral_conv2d_f64(x, w1, w2, modes1: int, modes2: int) -> np.ndarray:
    """Direct-DFT float64 restatement (C).  x [B,Cin,H,W]; w [Cin,Cout,m1,m2] complex."""
    x = _f32(x)
    w1 = _interleaved(w1)
    w2 = _interleaved(w2)
    B, Cin, H, W = x.shape
    Cout = w1.shape[1]
    y = np.empty((B, Cout, H, W), dtype=np.float64)
    rc = _load().oracle_spectral_conv2d(
        _ptr(x, ctypes.c_float), _ptr(w1, ctypes.c_float), _ptr(w2, ctypes.c_float),
        _ptr(y, ctypes.c_double), B, Cin, Cout, H, W, modes1, modes2)
    if rc != 0:
        raise ValueError(f"oracle_spectral_conv2d rejected the shape (rc={rc})")
    return y


def rfft2_corners_f64(x, modes1: int, modes2: int):
    """Corner spectra (float64, complex) of every plane: x [B,C,H,W] -> 2 x [B,C,m1,m2]."""
    x = _f32(x)
    B, C, H, W = x.shape
    x1 = np.empty((B, C, modes1, modes2, 2), dtype=np.float64)
    x2 = np.empty_like(x1)
    rc = _load().oracle_rfft2_corners(_ptr(x, ctypes.c_float), _ptr(x1, ctypes.c_double),
                                      _ptr(x2, ctypes.c_double), B * C, H, W, modes1, modes2)
    if rc != 0:
        raise ValueError(f"oracle_rfft2_corners rejected the shape (rc={rc})")
    return x1[..., 0] + 1j * x1[..., 1], x2[..., 0] + 1j * x2[..., 1]


def spectral_conv2d_np(x, w1, w2, modes1: int, modes2: int) -> np.ndarray:
    """numpy float64 FFT restatement of reference_pytorch.py:30-47."""
    x = np.asarray(x, dtype=np.float64)
    w1 = np.asarray(w1).astype(np.complex128)
    w2 = np.asarray(w2).astype(np.complex128)
    B, _, H, W = x.shape
    x_ft = np.fft.rfft2(x)
    out_ft = np.zeros((B, w1.shape[1], H, W // 2 + 1), dtype=np.complex128)
    out_ft[:, :, :modes1, :modes2] = np.einsum("bixy,ioxy->boxy", x_ft[:, :, :modes1, :modes2], w1)
    out_ft[:, :, -modes1:, :modes2] = np.einsum("bixy,ioxy->boxy", x_ft[:, :, -modes1:, :modes2], w2)
    return np.fft.irfft2(out_ft, s=(H, W))


def spectral_conv2d_torch(x, w1, w2, modes1: int, modes2: int):
    """The reference's CPU recipe (torch.fft + einsum, fp32/complex64) restated."""
    import torch

    x = torch.as_tensor(x, dtype=torch.float32)
    w1 = torch.as_tensor(w1).to(torch.complex64)
    w2 = torch.as_tensor(w2).to(torch.complex64)
    B, _, H, W = x.shape
    x_ft = torch.fft.rfft2(x)
    out_ft = torch.zeros(B, w1.shape[1], H, W // 2 + 1, dtype=torch.complex64)
    out_ft[:, :, :modes1, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, :modes1, :modes2], w1)
    out_ft[:, :, -modes1:, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, -modes1:, :modes2], w2)
    return torch.fft.irfft2(out_ft, s=(H, W))


def spectral_conv2d_grads_torch(x, w1, w2, modes1: int, modes2: int, grad_y):
    """Gradients of the reference recipe (``spectral_conv2d_torch``) by torch autograd in
    float64 / complex128: (grad_x, grad_w1, grad_w2) for the upstream gradient grad_y."""
    import torch

    x = torch.as_tensor(x).to(torch.float64).clone().requires_grad_(True)
    w1 = torch.as_tensor(w1).to(torch.complex128).clone().requires_grad_(True)
    w2 = torch.as_tensor(w2).to(torch.complex128).clone().requires_grad_(True)
    B, _, H, W = x.shape
    x_ft = torch.fft.rfft2(x)
    out_ft = torch.zeros(B, w1.shape[1], H, W // 2 + 1, dtype=torch.complex128)
    out_ft[:, :, :modes1, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, :modes1, :modes2], w1)
    out_ft[:, :, -modes1:, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, -modes1:, :modes2], w2)
    y = torch.fft.irfft2(out_ft, s=(H, W))
    y.backward(torch.as_tensor(grad_y).to(torch.float64))
    return x.grad, w1.grad, w2.grad


def spectral_conv3d_np(x, w, modes1: int, modes2: int, modes3: int) -> np.ndarray:
    """spectral_conv_combo/reference_pytorch.py:51-82 restated in numpy float64: rfftn over
    (D, H, W), the single corner [:m1, :m2, :m3] mixed per mode, zero-padded irfftn."""
    x = np.asarray(x, dtype=np.float64)
    w = np.asarray(w).astype(np.complex128)
    B, _, D, H, W = x.shape
    xf = np.fft.rfftn(x, axes=(-3, -2, -1))
    out = np.zeros((B, w.shape[1], D, H, W // 2 + 1), dtype=np.complex128)
    out[:, :, :modes1, :modes2, :modes3] = np.einsum("bixyz,ioxyz->boxyz", xf[:, :, :modes1, :modes2, :modes3], w)
    return np.fft.irfftn(out, s=(D, H, W), axes=(-3, -2, -1))


def spectral_conv3d_4c_np(x, ws, modes1: int, modes2: int, modes3: int) -> np.ndarray:
    """official_baseline.py:84-98 (four-corner SpectralConv3d.forward) restated in numpy
    float64: corners assigned in the baseline's order, later ones overwriting overlaps."""
    x = np.asarray(x, dtype=np.float64)
    ws = [np.asarray(w).astype(np.complex128) for w in ws]
    B, _, D, H, W = x.shape
    xf = np.fft.rfftn(x, axes=(-3, -2, -1))
    out = np.zeros((B, ws[0].shape[1], D, H, W // 2 + 1), dtype=np.complex128)
    sl1 = [slice(None, modes1), slice(D - modes1, None)]
    sl2 = [slice(None, modes2), slice(H - modes2, None)]
    for c, w in enumerate(ws):
        a, b = c & 1, c >> 1
        idx = (slice(None), slice(None), sl1[a], sl2[b], slice(None, modes3))
        out[idx] = np.einsum("bixyz,ioxyz->boxyz", xf[idx], w)
    return np.fft.irfftn(out, s=(D, H, W), axes=(-3, -2, -1))


def fno2d_torch(state: dict, x, *, n_layers: int = 4, modes1: int = 12, modes2: int = 12,
                instance_norm: bool = True, dtype=None):
    """Restatement of FNO2d.forward(use_supa=False) (fno_ns/model.py:183-198).

    ``state`` is an FNO2d state dict (parameter names of fno_ns/model.py:158-166, 92-94);
    ``x`` is [B, T_in, H, W] (the grid channels are appended here, model.py:168-181, 193-194).
    ``instance_norm=False`` gives the norm-free layer of the benchmark text
    (SpectralConv + 1x1 skip + GELU).  ``dtype`` (default float32) sets the arithmetic.
    """
    import torch
    import torch.nn.functional as F

    dtype = dtype or torch.float32
    cdtype = torch.complex128 if dtype == torch.float64 else torch.complex64
    st = {k: torch.as_tensor(v) for k, v in state.items()}
    x = torch.as_tensor(x).to(dtype)
    B, _, H, W = x.shape
    gx = torch.linspace(0, 1, H, dtype=torch.float32).to(dtype).reshape(1, 1, H, 1).expand(B, 1, H, W)
    gy = torch.linspace(0, 1, W, dtype=torch.float32).to(dtype).reshape(1, 1, 1, W).expand(B, 1, H, W)
    h = torch.cat([x, gx, gy], dim=1)

    def conv1x1(t, w, b):
        return F.conv2d(t, w.to(dtype), b.to(dtype))

    h = conv1x1(h, st["lift.weight"], st["lift.bias"])
    for i in range(n_layers):
        p = f"fourier_layers.{i}."
        w1 = st[p + "spectral_conv.weights1"].to(cdtype)
        w2 = st[p + "spectral_conv.weights2"].to(cdtype)
        x_ft = torch.fft.rfft2(h)
        out_ft = torch.zeros(B, w1.shape[1], H, W // 2 + 1, dtype=cdtype)
        out_ft[:, :, :modes1, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, :modes1, :modes2], w1)
        out_ft[:, :, -modes1:, :modes2] = torch.einsum("bixy,ioxy->boxy", x_ft[:, :, -modes1:, :modes2], w2)
        spectral = torch.fft.irfft2(out_ft, s=(H, W))
        z = spectral + conv1x1(h, st[p + "conv.weight"], st[p + "conv.bias"])
        if instance_norm:
            z = F.instance_norm(z, eps=1e-5)
        h = F.gelu(z)
    h = F.gelu(conv1x1(h, st["project.0.weight"], st["project.0.bias"]))
    return conv1x1(h, st["project.2.weight"], st["project.2.bias"])


def rel_errors(expected, actual) -> tuple[float, float]:
    """(Frobenius relative error, max-abs / max|ref|): the two metrics of
    spectral_conv_combo/test_accuracy.py:22-27 and test_irregular_shapes.py:78-80."""
    e = np.asarray(expected, dtype=np.float64)
    a = np.asarray(actual, dtype=np.float64)
    ref_norm = np.linalg.norm(e)
    diff = np.linalg.norm(e - a)
    fro = diff if ref_norm < 1e-12 else diff / ref_norm
    mx = np.abs(e - a).max() / max(np.abs(e).max(), 1e-9)
    return float(fro), float(mx)


def threads() -> int:
    return os.cpu_count() or 1
