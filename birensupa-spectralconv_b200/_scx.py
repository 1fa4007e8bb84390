"""ctypes binding of libscx.so, the C-ABI device library (include/scx.h).

The library is required: importing this module without the built ``libscx.so`` raises
ImportError, and every call on a CPU-only machine fails with the CUDA status the library
returns.  There is no host fallback.
"""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
LIB_PATH = PKG_DIR / "libscx.so"
HEADER_PATH = PKG_DIR.parent / "include" / "scx.h"

if not LIB_PATH.exists():
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C {PKG_DIR}` (or __graft_entry__.build())")

lib = ctypes.CDLL(str(LIB_PATH))

_i = ctypes.c_int
_p = ctypes.c_void_p
_sz = ctypes.c_size_t


class FnoConfig(ctypes.Structure):
    _fields_ = [
        ("batch_size", _i), ("height", _i), ("width", _i), ("in_frames", _i),
        ("input_layout", _i), ("hidden", _i), ("modes1", _i), ("modes2", _i),
        ("n_layers", _i), ("proj_hidden", _i), ("out_channels", _i), ("instance_norm", _i),
    ]


MAX_LAYERS = 16


class FnoParams(ctypes.Structure):
    _fields_ = [
        ("lift_w", _p), ("lift_b", _p),
        ("spectral_w1", _p * MAX_LAYERS), ("spectral_w2", _p * MAX_LAYERS),
        ("skip_w", _p * MAX_LAYERS), ("skip_b", _p * MAX_LAYERS),
        ("proj1_w", _p), ("proj1_b", _p), ("proj2_w", _p), ("proj2_b", _p),
    ]


_SIGNATURES = {
    "scx_version": ([], _i),
    "scx_status_string": ([_i], ctypes.c_char_p),
    "scx_prepare": ([_i, _i, _i, _i], _i),
    "scx_watchdog": ([_i], _i),
    "scx_spectral_mul": ([_p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "scx_spectral_mul_dual": ([_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p], _i),
    "scx_spectral_mul_bwd_workspace_size": ([_i, _i, _i, _i, _i], _sz),
    "scx_spectral_mul_bwd": ([_p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "scx_rfft2_corners": ([_p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "scx_irfft2_corners": ([_p, _p, _p, _i, _i, _i, _i, _i, _i, _p], _i),
    "scx_rfft2": ([_p, _p, _i, _i, _i, _i, _p], _i),
    "scx_irfft2": ([_p, _p, _i, _i, _i, _i, _p], _i),
    "scx_spectral_conv2d_workspace_size": ([_i, _i, _i, _i, _i, _i, _i], _sz),
    "scx_spectral_conv2d_fwd": ([_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "scx_spectral_conv2d_fwd_noalloc": ([_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p], _i),
    "scx_spectral_conv3d_workspace_size": ([_i, _i, _i, _i, _i, _i, _i, _i, _i], _sz),
    "scx_spectral_conv3d_fwd": ([_p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "scx_spectral_conv3d_4c_workspace_size": ([_i, _i, _i, _i, _i, _i, _i, _i, _i], _sz),
    "scx_spectral_conv3d_4c_fwd": ([_p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "scx_spectral_conv2d_bwd_workspace_size": ([_i, _i, _i, _i, _i, _i, _i], _sz),
    "scx_spectral_conv2d_bwd": ([_p, _p, _p, _p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _sz, _p], _i),
    "scx_spectral_conv2d_fwd_host": ([_p, _p, _p, _p, _i, _i, _i, _i, _i, _i, _i, _p, _p, _p, _sz, _i, _p], _i),
    "scx_dft_variants": ([_i, _i, _i, _i], _i),
    "scx_set_dft_variant": ([_i, _i, _i, _i, _i], _i),
    "scx_set_mix_variant": ([_i, _i, _i, _i, _i, _i], _i),
    "scx_get_variant": ([_i, _i, _i, _i, _i, _i], _i),
    "scx_clear_variants": ([], None),
    "scx_fno2d_workspace_size": ([ctypes.POINTER(FnoConfig)], _sz),
    "scx_fno2d_fwd": ([ctypes.POINTER(FnoConfig), ctypes.POINTER(FnoParams), _p, _p, _p, _sz, _p], _i),
    "scx_ipc_handle_bytes": ([], _i),
    "scx_ipc_export": ([_p, _p, ctypes.POINTER(ctypes.c_ulonglong)], _i),
    "scx_ipc_import": ([_p, ctypes.POINTER(ctypes.c_void_p)], _i),
    "scx_ipc_close": ([_p], _i),
    "scx_copy_async": ([_p, _p, _sz, _p], _i),
}

for _name, (_args, _ret) in _SIGNATURES.items():
    if hasattr(lib, _name):
        _fn = getattr(lib, _name)
        _fn.argtypes = _args
        _fn.restype = _ret


def header_symbols() -> list[str]:
    """Every function declared in include/scx.h."""
    text = HEADER_PATH.read_text()
    return sorted(set(re.findall(r"^\s*(?:[\w\s\*]+?)\b(scx_\w+)\s*\(", text, flags=re.M)))


def check(status: int, what: str) -> None:
    if status != 0:
        name = lib.scx_status_string(status)
        raise RuntimeError(f"{what} failed with CUDA status {status} ({name.decode() if name else '?'})")


def stream_of(device: torch.device) -> int:
    return torch.cuda.current_stream(device).cuda_stream


def ptr(t: torch.Tensor) -> int:
    return t.data_ptr()


class device_guard:
    """Makes ``device`` current for the C calls (they act on the current device)."""

    def __init__(self, device: torch.device):
        self.idx = device.index if device.index is not None else torch.cuda.current_device()
        self.prev = None

    def __enter__(self):
        cur = torch.cuda.current_device()
        if cur != self.idx:
            self.prev = cur
            torch.cuda.set_device(self.idx)
        return self

    def __exit__(self, *exc):
        if self.prev is not None:
            torch.cuda.set_device(self.prev)
        return False
