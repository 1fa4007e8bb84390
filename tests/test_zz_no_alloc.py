"""GPU: the allocation-free entry point scx_spectral_conv2d_fwd_noalloc, called through
the C ABI, matches the regular scx_spectral_conv2d_fwd on two calls in a row.

The allocation-free variant serves callers that cannot let the library call cudaMalloc
(for example a process whose memory pool already owns the GPU memory); it keeps its
spectra and twiddle tables in a fixed 16 MiB device array instead of a caller workspace
and the library's twiddle cache.  This file is collected last on purpose."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import _scx
import scx_data
from oracle import oracle

pytestmark = pytest.mark.gpu

TOL = 1e-4
OOM = 2  # cudaErrorMemoryAllocation: the shape needs more than the fixed scratch


def _inputs(name, device):
    x, w1, w2, c = scx_data.make_spectral_case(name)
    return (x.to(device), torch.view_as_real(w1.to(device)).contiguous(),
            torch.view_as_real(w2.to(device)).contiguous(), c)


def _noalloc(x, w1, w2, c, y, stream):
    return _scx.lib.scx_spectral_conv2d_fwd_noalloc(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(),
                                                    c["B"], c["Cin"], c["Cout"], c["H"], c["W"], c["m1"], c["m2"],
                                                    stream)


def _regular(x, w1, w2, c, stream):
    y = torch.empty(c["B"], c["Cout"], c["H"], c["W"], device=x.device)
    nbytes = _scx.lib.scx_spectral_conv2d_workspace_size(c["B"], c["Cin"], c["Cout"], c["H"], c["W"], c["m1"],
                                                         c["m2"])
    ws = torch.empty(nbytes, dtype=torch.uint8, device=x.device)
    rc = _scx.lib.scx_spectral_conv2d_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), c["B"],
                                          c["Cin"], c["Cout"], c["H"], c["W"], c["m1"], c["m2"], ws.data_ptr(),
                                          nbytes, stream)
    assert rc == 0, rc
    return y


def test_noalloc_matches_regular_entry_point_two_calls(cuda_device):
    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    results = []
    # two calls in a row with different shapes: the second must not see the first's leftovers
    for name in ("spectral_b20_c32_128x128_m16_grf", "spectral_b7_c20to36_96x160_m16x20"):
        x, w1, w2, c = _inputs(name, cuda_device)
        y_na = torch.full((c["B"], c["Cout"], c["H"], c["W"]), float("nan"), device=cuda_device)
        assert _noalloc(x, w1, w2, c, y_na, stream) == 0
        results.append((name, x, w1, w2, c, y_na))
    torch.cuda.synchronize(cuda_device)
    for name, x, w1, w2, c, y_na in results:
        y_reg = _regular(x, w1, w2, c, stream)
        torch.cuda.synchronize(cuda_device)
        got = y_na.cpu().numpy()
        assert np.isfinite(got).all(), name
        fro, mx = oracle.rel_errors(y_reg.cpu().numpy(), got)
        assert fro <= TOL and mx <= TOL, (name, fro, mx)


def test_noalloc_rejects_shapes_beyond_the_scratch(cuda_device):
    torch.cuda.set_device(cuda_device)
    stream = torch.cuda.current_stream(cuda_device).cuda_stream
    B, Cin, Cout, H, W, m1, m2 = 16, 64, 64, 64, 64, 32, 32  # ~34 MB of spectra > 16 MiB
    x = torch.zeros(B, Cin, H, W, device=cuda_device)
    w = torch.zeros(Cin, Cout, m1, m2, 2, device=cuda_device)
    y = torch.full((B, Cout, H, W), 7.0, device=cuda_device)
    rc = _scx.lib.scx_spectral_conv2d_fwd_noalloc(x.data_ptr(), w.data_ptr(), w.data_ptr(), y.data_ptr(), B, Cin,
                                                  Cout, H, W, m1, m2, stream)
    assert rc == OOM
    torch.cuda.synchronize(cuda_device)
    assert bool((y == 7.0).all())  # nothing was launched
