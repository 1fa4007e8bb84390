"""GPU: the allocation-free entry point scx_spectral_conv2d_fwd_noalloc, called through
the C ABI, matches the regular scx_spectral_conv2d_fwd on two calls in a row.

The allocation-free variant serves callers that cannot let the library call cudaMalloc
(for example a process whose memory pool already owns the GPU memory); it keeps its
spectra and twiddle tables in a fixed 16 MiB device array instead of a caller workspace
and the library's twiddle cache.  This file is collected last, so that a run stopping at
its first failure has run every other test; the claim that the entry point allocates
nothing is checked in a fresh child process whose first libscx call is the allocation-free
one (``test_noalloc_first_call_in_fresh_process``), so it does not depend on that order."""

from __future__ import annotations

import json
import os
import shutil
import subprocess
import sys
from pathlib import Path

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


_CHILD = r"""
import ctypes, json, sys
import torch
probe = ctypes.CDLL(sys.argv[1])
dev = torch.device("cuda", 0)
torch.cuda.set_device(dev)
import scx_data
cases = []
for name in ("spectral_b20_c32_128x128_m16_grf", "spectral_b7_c20to36_96x160_m16x20"):
    x, w1, w2, c = scx_data.make_spectral_case(name)
    cases.append((x.to(dev), torch.view_as_real(w1.to(dev)).contiguous(),
                  torch.view_as_real(w2.to(dev)).contiguous(), c,
                  torch.full((c["B"], c["Cout"], c["H"], c["W"]), float("nan"), device=dev)))
ws = torch.empty(64 << 20, dtype=torch.uint8, device=dev)  # workspace of the regular call, made up front
torch.cuda.synchronize(dev)
import _scx  # first load of libscx.so in this process
lib = _scx.lib
stream = torch.cuda.current_stream(dev).cuda_stream
before = (probe.alloc_probe_mallocs(), probe.alloc_probe_memcpys())
rcs = []
for x, w1, w2, c, y in cases:  # the first libscx calls of the process: allocation-free
    rcs.append(lib.scx_spectral_conv2d_fwd_noalloc(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(),
                                                   c["B"], c["Cin"], c["Cout"], c["H"], c["W"], c["m1"], c["m2"],
                                                   stream))
torch.cuda.synchronize(dev)
after = (probe.alloc_probe_mallocs(), probe.alloc_probe_memcpys())
finite = [bool(torch.isfinite(y).all()) for *_, y in cases]
x, w1, w2, c, y = cases[0]
need = lib.scx_spectral_conv2d_workspace_size(c["B"], c["Cin"], c["Cout"], c["H"], c["W"], c["m1"], c["m2"])
rc_reg = lib.scx_spectral_conv2d_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), c["B"], c["Cin"],
                                     c["Cout"], c["H"], c["W"], c["m1"], c["m2"], ws.data_ptr(), need, stream)
torch.cuda.synchronize(dev)
regular = (probe.alloc_probe_mallocs(), probe.alloc_probe_memcpys())
print(json.dumps({"rcs": rcs, "before": before, "after": after, "finite": finite, "rc_regular": rc_reg,
                  "regular": regular, "watchdog": lib.scx_watchdog(0)}))
"""


def test_noalloc_first_call_in_fresh_process(tmp_path):
    """In a new process whose first libscx.so calls are two allocation-free forwards, the
    library makes no cudaMalloc and no blocking cudaMemcpy (counted by a preloaded probe that
    sees every such call made from libscx.so).  The regular entry point called afterwards
    in the same process does allocate (its first use of a shape builds the twiddle tables),
    which shows that the probe sees the library's calls."""
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    gcc = shutil.which("gcc") or shutil.which("cc")
    if gcc is None:
        pytest.skip("no C compiler for the probe")
    here = Path(__file__).resolve().parent
    probe = tmp_path / "alloc_probe.so"
    subprocess.run([gcc, "-shared", "-fPIC", "-O1", "-o", str(probe), str(here / "alloc_probe.c"), "-ldl",
                    f"-Wl,--version-script={here / 'alloc_probe.map'}"], check=True)
    env = dict(os.environ)
    env["LD_PRELOAD"] = str(probe)
    repo = here.parent
    env["PYTHONPATH"] = os.pathsep.join([str(repo / "birensupa-spectralconv_b200"), str(repo),
                                         env.get("PYTHONPATH", "")])
    out = subprocess.run([sys.executable, "-c", _CHILD, str(probe)], env=env, capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-4000:]
    r = json.loads(out.stdout.strip().splitlines()[-1])
    assert r["rcs"] == [0, 0], r
    assert r["after"] == r["before"] == [0, 0], r  # no cudaMalloc, no blocking copy
    assert all(r["finite"]), r
    assert r["rc_regular"] == 0 and r["regular"][0] > r["after"][0], r
    assert r["watchdog"] == 0, r
