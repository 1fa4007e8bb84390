"""GPU parity of the FNO-2d forward (fno_ns/model.py) through libscx.so's fused entry
point, against the reference's golden output and the oracle restatement.  Tolerance
1e-4 on both the Frobenius and the max-abs relative error, as for SpectralConv2d."""

from __future__ import annotations

import numpy as np
import pytest
import torch

import scx_data
from conftest import load_golden
from oracle import oracle
from test_oracle import check_against_golden, fno_state

pytestmark = pytest.mark.gpu
TOL = 1e-4


def _close(ref, got, tol=TOL):
    fro, mx = oracle.rel_errors(ref, got)
    assert fro <= tol and mx <= tol, f"frobenius rel {fro:.3e}, max-abs rel {mx:.3e}"


def test_fno_matches_reference_golden(cuda_device):
    g = load_golden("fno_fno_ns_b20_w32_64x64_m12_l4.npz")
    model = fno_state(int(g["init_seed"])).to(cuda_device)
    fw = scx_data.FNO_WORKLOAD
    x_cl = scx_data.fno_input(fw["B"], fw["seed"], H=fw["H"], W=fw["W"], frames=fw["frames"])
    # channels-last [B, H, W, T+2] input (frames + grid), the benchmark's layout
    y_cl = model.forward_device(x_cl.to(cuda_device), channels_last=True)
    # reference layout [B, T, H, W], grid generated inside
    x = x_cl[..., : fw["frames"]].permute(0, 3, 1, 2).contiguous()
    y = model.forward_device(x.to(cuda_device))
    torch.cuda.synchronize(cuda_device)
    for out in (y_cl, y):
        got = out.cpu().numpy()
        assert np.isfinite(got).all()
        check_against_golden(g, got, TOL)
    ref = oracle.fno2d_torch(model.cpu().state_dict(), x)
    _close(ref.numpy(), y.cpu().numpy())
    # reference-facing call: host in, host out
    host = model.to(cuda_device).forward(x)
    assert host.device.type == "cpu"
    check_against_golden(g, host.numpy(), TOL)


@pytest.mark.parametrize("cfg", [
    dict(B=3, T=6, H=32, W=48, width=16, m1=8, m2=10, layers=4, norm=True),
    dict(B=2, T=10, H=40, W=40, width=24, m1=24, m2=21, layers=5, norm=False),  # overlap + Nyquist
    dict(B=1, T=3, H=17, W=23, width=8, m1=5, m2=7, layers=4, norm=True),       # odd sizes
    dict(B=2, T=4, H=88, W=88, width=32, m1=10, m2=12, layers=4, norm=True),    # 8-CTA cluster, partial CTA
    dict(B=2, T=4, H=96, W=96, width=16, m1=8, m2=8, layers=4, norm=True),      # plane too large for a cluster
    dict(B=2, T=5, H=32, W=32, width=32, m1=8, m2=8, layers=4, norm=False),     # four-pixel skip with GELU
    dict(B=3, T=4, H=32, W=32, width=32, m1=8, m2=8, layers=4, norm=True),      # pixel tiles, 4-CTA cluster
    dict(B=2, T=4, H=16, W=16, width=32, m1=4, m2=5, layers=4, norm=True),      # pixel tiles, one CTA per plane
    dict(B=1, T=10, H=64, W=64, width=32, m1=12, m2=12, layers=4, norm=True),   # pixel tiles, 16-CTA cluster
])
def test_fno_shapes_vs_oracle(cfg, cuda_device):
    import fno_model

    torch.manual_seed(123)
    model = fno_model.FNO2d(modes1=cfg["m1"], modes2=cfg["m2"], width=cfg["width"], n_layers=cfg["layers"],
                            in_channels=cfg["T"], instance_norm=cfg["norm"])
    x = scx_data.gaussian((cfg["B"], cfg["T"], cfg["H"], cfg["W"]), 5)
    ref = oracle.fno2d_torch(model.state_dict(), x, n_layers=cfg["layers"], modes1=cfg["m1"], modes2=cfg["m2"],
                             instance_norm=cfg["norm"])
    y = model.to(cuda_device).forward_device(x.to(cuda_device))
    _close(ref.detach().numpy(), y.cpu().numpy())


def test_fno_cuda_graph_replay_is_identical(cuda_device):
    """The whole forward is capturable: replaying a graph gives the eager result bitwise."""
    model = fno_state(0).to(cuda_device)
    fw = scx_data.FNO_WORKLOAD
    x_cl = scx_data.fno_input(4, 9, H=fw["H"], W=fw["W"], frames=fw["frames"]).to(cuda_device)
    eager = model.forward_device(x_cl, channels_last=True).clone()   # also warms the caches
    static_out = torch.empty_like(eager)
    torch.cuda.synchronize(cuda_device)
    graph = torch.cuda.CUDAGraph()
    s = torch.cuda.Stream(cuda_device)
    s.wait_stream(torch.cuda.current_stream(cuda_device))
    with torch.cuda.stream(s):
        model.forward_device(x_cl, channels_last=True, out=static_out)
    torch.cuda.current_stream(cuda_device).wait_stream(s)
    with torch.cuda.graph(graph):
        model.forward_device(x_cl, channels_last=True, out=static_out)
    static_out.zero_()
    graph.replay()
    torch.cuda.synchronize(cuda_device)
    assert torch.equal(static_out, eager)
    del graph


def test_fno_rejects_bad_inputs(cuda_device):
    model = fno_state(0).to(cuda_device)
    with pytest.raises(ValueError):
        model.forward_device(torch.zeros(2, 9, 64, 64, device=cuda_device))          # wrong frame count
    with pytest.raises(ValueError):
        model.forward_device(torch.zeros(2, 64, 64, 11, device=cuda_device), channels_last=True)
    with pytest.raises(RuntimeError):
        model.forward_device(torch.zeros(2, 10, 64, 64))                              # host tensor
