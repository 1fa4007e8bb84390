"""GPU: the batch-sharded CUDA path gives the single-GPU result.

* One GPU: contiguous (ragged) batch shards run one after another through the public API
  give the same output as the whole batch in one call.
* Two or more GPUs (skipped otherwise): one process per GPU under torchrun, NCCL; each rank
  runs its shard on its own GPU, the shards are gathered into a preallocated tensor on rank 0
  (scx_dist.gather_batch_into), and rank 0 compares them with the whole batch run alone on its
  GPU; the peer-copy gather (scx_dist.PeerGather) must give the NCCL gather's bits, and the
  overlapped form (scx_dist.PipelinedGather: sub-batch forwards, each pushed while the next is
  computed) the single-GPU result to the same tolerance.

Per plane the transforms are computed the same way whatever the batch; the mixing kernel's
tile shape is chosen per batch size and may split the channel sum into a different number of
partial sums (a B=7 shard takes another tile shape than B=20), so the bound is 1e-5 of max|y|
(observed: up to 3.3e-6) rather than bitwise equality."""

from __future__ import annotations

import json
import os
import socket
import subprocess
import sys
from pathlib import Path

import pytest
import torch

import scx_data
import scx_dist

pytestmark = pytest.mark.gpu

REPO = Path(__file__).resolve().parents[1]
TOL = 1e-5


def _run(x, w1, w2, m1, m2, device):
    import spectral_conv_ops

    y = spectral_conv_ops.spectral_conv2d_supa(x.to(device), w1.to(device), w2.to(device), m1, m2,
                                               use_sufft="fused", to_cpu=False)
    torch.cuda.synchronize(device)
    return y


@pytest.mark.parametrize("name,world", [("spectral_b20_c32_128x128_m16_grf", 8),
                                        ("spectral_b20_c32_64x64_m12", 3),
                                        ("spectral_b16_c64_256x256_m32", 8),
                                        ("spectral_b7_c20to36_96x160_m16x20", 4)])
def test_shards_on_one_gpu_equal_whole_batch(name, world, cuda_device):
    x, w1, w2, c = scx_data.make_spectral_case(name)
    whole = _run(x, w1, w2, c["m1"], c["m2"], cuda_device)
    parts = [_run(x[lo:hi].contiguous(), w1, w2, c["m1"], c["m2"], cuda_device)
             for lo, hi in (scx_dist.shard_range(c["B"], world, r) for r in range(world))]
    sharded = torch.cat(parts)
    scale = whole.abs().max().item()
    assert (sharded - whole).abs().max().item() <= TOL * scale


_CHILD = r"""
import json, os, sys
import torch
import scx_data, scx_dist
import spectral_conv_ops
rank, local, world = scx_dist.env_rank()
dev = torch.device("cuda", local)
torch.cuda.set_device(dev)
os.environ["NCCL_NVLS_ENABLE"] = "0"
scx_dist.init("nccl", timeout_s=60, device=dev)
name = sys.argv[1]
x, w1, w2, c = scx_data.make_spectral_case(name)
B = c["B"]
lo, hi = scx_dist.shard_range(B, world, rank)
y = spectral_conv_ops.spectral_conv2d_supa(x[lo:hi].contiguous().to(dev), w1.to(dev), w2.to(dev), c["m1"], c["m2"],
                                           use_sufft="fused", to_cpu=False)
out = torch.empty((B,) + tuple(y.shape[1:]), device=dev) if rank == 0 else None
scx_dist.gather_batch_into(y.contiguous(), out, B)
torch.cuda.synchronize(dev)
if rank == 0:
    whole = spectral_conv_ops.spectral_conv2d_supa(x.to(dev), w1.to(dev), w2.to(dev), c["m1"], c["m2"],
                                                   use_sufft="fused", to_cpu=False)
    torch.cuda.synchronize(dev)
    scale = whole.abs().max().item()
# the same gather by peer copies (CUDA IPC) into a NaN-poisoned output, twice
out2 = torch.full((B,) + tuple(y.shape[1:]), float("nan"), device=dev) if rank == 0 else None
peer = scx_dist.PeerGather(y.contiguous(), out2, B)
for _ in range(2):
    peer.push(torch.cuda.current_stream(dev).cuda_stream)
peer.sync()
peer.close()
# the overlapped form: sub-batch forwards, each pushed while the next is computed, twice
out3 = torch.full((B,) + tuple(y.shape[1:]), float("nan"), device=dev) if rank == 0 else None
y3 = out3[lo:hi] if rank == 0 else torch.empty_like(y)
pipe = scx_dist.PipelinedGather(x[lo:hi].contiguous().to(dev), y3, torch.view_as_real(w1.to(dev)).contiguous(),
                                torch.view_as_real(w2.to(dev)).contiguous(), c["m1"], c["m2"], out3, B)
for _ in range(2):
    pipe.run(torch.cuda.current_stream(dev))
pipe.peer.sync()
pipe.close()
if rank == 0:
    print(json.dumps({"rel": (out - whole).abs().max().item() / scale, "bitwise": bool(torch.equal(out, whole)),
                      "peer_equal": bool(torch.equal(out2, out)),
                      "pipe_rel": (out3 - whole).abs().max().item() / scale}))
torch.distributed.barrier()
torch.distributed.destroy_process_group()
"""


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.parametrize("name", ["spectral_b20_c32_128x128_m16_grf", "spectral_b16_c64_256x256_m32"])
def test_nccl_sharded_equals_single_gpu(name, tmp_path):
    n = torch.cuda.device_count()
    if n < 2:
        pytest.skip("needs two GPUs")
    world = min(n, 4)
    script = tmp_path / "child.py"
    script.write_text(_CHILD)
    env = dict(os.environ)
    env["PYTHONPATH"] = os.pathsep.join([str(REPO / "birensupa-spectralconv_b200"), str(REPO),
                                         env.get("PYTHONPATH", "")])
    env["NCCL_NVLS_ENABLE"] = "0"
    cmd = ["timeout", "-k", "30", "240", sys.executable, "-m", "torch.distributed.run", "--nnodes=1",
           f"--nproc-per-node={world}", "--master-addr=127.0.0.1", f"--master-port={_free_port()}", str(script), name]
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-4000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    r = json.loads(lines[-1])
    assert r["rel"] <= TOL, r
    assert r["peer_equal"], r
    assert r["pipe_rel"] <= TOL, r  # NaN (a slot never written) fails too
