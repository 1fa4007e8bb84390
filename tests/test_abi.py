"""CPU: the C-ABI library loads, exports every symbol include/scx.h declares, and rejects
invalid arguments with cudaErrorInvalidValue before touching a device."""

from __future__ import annotations

import ctypes

import pytest

import _scx

INVALID = 1  # cudaErrorInvalidValue


def test_every_header_symbol_is_exported():
    symbols = _scx.header_symbols()
    assert "scx_spectral_conv2d_fwd" in symbols and "scx_spectral_mul_dual" in symbols
    missing = [s for s in symbols if not hasattr(_scx.lib, s)]
    assert not missing, missing


def test_version_and_status_strings():
    assert _scx.lib.scx_version() >= 100
    assert _scx.lib.scx_status_string(0)
    assert _scx.lib.scx_status_string(INVALID)


def test_workspace_size_formula():
    ws = _scx.lib.scx_spectral_conv2d_workspace_size
    assert ws(20, 32, 32, 64, 64, 12, 12) == 2 * (20 * 32 * 144 + 20 * 32 * 144) * 8
    assert ws(7, 20, 36, 96, 160, 16, 20) == 2 * (7 * 20 * 320 + 7 * 36 * 320) * 8
    assert ws(1, 1, 1, 8, 8, 9, 2) == 0      # m1 > H
    assert ws(1, 1, 1, 8, 8, 2, 6) == 0      # m2 > W//2+1
    assert ws(0, 1, 1, 8, 8, 2, 2) == 0


@pytest.mark.parametrize("args", [
    (0, 1, 1, 1, 1),      # batch 0
    (1, 0, 1, 1, 1),
    (1, 1, -1, 1, 1),
    (1, 1, 1, 0, 1),
])
def test_spectral_mul_rejects_sizes(args):
    p = ctypes.c_void_p(16)
    assert _scx.lib.scx_spectral_mul(p, p, p, *args, None) == INVALID
    assert _scx.lib.scx_spectral_mul_dual(p, p, p, p, p, p, *args, None) == INVALID


def test_null_and_misaligned_pointers_rejected():
    p = ctypes.c_void_p(256)
    assert _scx.lib.scx_spectral_mul(None, p, p, 1, 1, 1, 1, 1, None) == INVALID
    assert _scx.lib.scx_spectral_mul(ctypes.c_void_p(260), p, p, 1, 1, 1, 1, 1, None) == INVALID
    assert _scx.lib.scx_rfft2_corners(p, None, p, 1, 1, 8, 8, 2, 2, None) == INVALID
    assert _scx.lib.scx_spectral_conv2d_fwd(p, p, p, p, 1, 1, 1, 8, 8, 2, 2, None, 4096, None) == INVALID


def test_shape_rules_rejected():
    p = ctypes.c_void_p(256)
    assert _scx.lib.scx_rfft2_corners(p, p, p, 1, 1, 8, 8, 9, 2, None) == INVALID   # m1 > H
    assert _scx.lib.scx_rfft2_corners(p, p, p, 1, 1, 8, 8, 2, 6, None) == INVALID   # m2 > W//2+1
    assert _scx.lib.scx_irfft2_corners(p, p, p, 1, 1, 0, 8, 1, 1, None) == INVALID
    assert _scx.lib.scx_prepare(8, 8, 0, 1) == INVALID
    # workspace too small
    assert _scx.lib.scx_spectral_conv2d_fwd(p, p, p, p, 1, 1, 1, 8, 8, 2, 2, p, 8, None) == INVALID
