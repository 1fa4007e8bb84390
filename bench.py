#!/usr/bin/env python3
"""Benchmark of the B200 SpectralConv2d / FNO-NS forward.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload NAME]

One process per GPU (torchrun for N > 1, NCCL).  The headline workload is the
SpectralConv2d forward at B=20 per GPU, Cin=Cout=32, 128x128, modes 16 on a Gaussian
random field; the batch is sharded across GPUs (weak scaling: 20 items per GPU, no
collective on the data path).  ``value`` = samples processed by all ranks / max-over-ranks
device time of exactly K steps (CUDA events, after W warm-up steps).  Between timed steps
the inputs rotate over enough buffer sets that every step reads data larger than L2.

Rank 0 prints ONE JSON line.  Besides the contract keys it carries
* ``roofline``: the dominant kernel's algorithmic bytes per launch / its CUDA-event
  duration against the measured HBM copy bandwidth, and ``roofline_fused_path`` for the
  whole forward (x read + y written + both weight tensors read);
* ``e2e``: the same metric through the public host API (``spectral_conv2d_supa`` with a
  pinned host input and a host result), H2D and D2H inside the timed region;
* ``cpu_baseline``: the reference's CPU recipe (torch.fft + einsum, all host threads) on
  the same workload (rank 0, N=1);
* ``workloads``: the 64x64 and 256x256 SpectralConv2d forwards measured the same way, and
  the FNO-NS forward (B=20 per GPU, samples/s, NCCL output gather included when N > 1).

``--impl reference`` times the reference's CPU implementation of the path (its torch.fft
+ einsum recipe restated in ``oracle/``) on this host's cores, same workload and metric.
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import time
from pathlib import Path

REPO = Path(__file__).resolve().parent
PKG = REPO / "birensupa-spectralconv_b200"
sys.path.insert(0, str(PKG))
sys.path.insert(0, str(REPO))

import torch  # noqa: E402

HEADLINE = "spectral_b20_c32_128x128_m16_grf"
EXTRA_WORKLOADS = ["spectral_b20_c32_64x64_m12", "spectral_b16_c64_256x256_m32"]
IRREGULAR_WORKLOADS = ["spectral_b7_c20to36_96x160_m16x20", "spectral_b3_c24_100x72_m10",
                       "spectral_b1_c48_130x130_m24"]
STRONG_WORKLOAD = "spectral_b16_c64_256x256_m32"  # B=16 in total, sharded over the ranks
L2_BYTES = 126 * 1024 * 1024
FALLBACK_HBM_GBS = 6650.0


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--workload", default=HEADLINE)
    ap.add_argument("--no-extras", action="store_true", help="skip every extra workload")
    ap.add_argument("--extras", default="all",
                    help="comma list of extra workloads to run: 64, 256, irr, c3s, fno, bwd (default: all)")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    return ap.parse_args()


# ----------------------------------------------------------------------------- helpers

def hbm_peak() -> tuple[float, str]:
    p = REPO / "MEASURED_PEAKS.json"
    try:
        v = float(json.loads(p.read_text())["hbm_gbs"])
        return v, "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def spectral_bytes(c: dict) -> dict:
    """Algorithmic HBM bytes: every operand read once, every result written once."""
    B, Cin, Cout, H, W, m1, m2 = (c[k] for k in ("B", "Cin", "Cout", "H", "W", "m1", "m2"))
    nm = m1 * m2
    return {
        "dft_fwd": 4 * B * Cin * H * W + 16 * B * Cin * nm,
        "mix": 16 * B * Cin * nm + 16 * Cin * Cout * nm + 16 * B * Cout * nm,
        "dft_inv": 16 * B * Cout * nm + 4 * B * Cout * H * W,
        "fused_path": 4 * B * H * W * (Cin + Cout) + 16 * Cin * Cout * nm,
    }


def launches_per_forward(c: dict) -> int:
    """Kernel launches of one scx_spectral_conv2d_fwd, by the library's dispatch rule: three
    (forward DFT, mixing, inverse DFT; at 256 x 256 the forward folds its four parity
    sub-problems in one launch and the inverse computes the four output quadrants in one), or
    seven when another plane with a 256-point side runs folded (the folding forward, mixing,
    four inverse sub-transforms, unfold)."""
    def direct(H, W, m1, m2):  # tc_fwd_supported
        return (H in (64, 128) and W in (64, 128) and 1 <= m1 and 2 * m1 <= 32 and 1 <= m2 <= 32 and m1 <= H
                and m2 <= W // 2 + 1)

    H, W, m1, m2 = c["H"], c["W"], c["m1"], c["m2"]
    split = (H in (128, 256) and W in (128, 256) and m1 % 2 == 0 and m2 % 2 == 0 and 2 * m1 <= H
             and m1 >= 2 and m2 >= 2 and direct(H // 2, W // 2, m1 // 2, m2 // 2))
    quad = H == 256 and W == 256 and 1 <= m1 <= 32 and 1 <= m2 <= 32  # tc_quad_supported
    return 7 if split and not direct(H, W, m1, m2) and not quad else 3


def fixture_error(name: str, y: torch.Tensor, prefix: str = "spectral", ref: str = "reference_pytorch.py") -> dict | None:
    """Error of a device result against the reference's output for the same workload, as
    committed in tests/golden (4096 sampled outputs, per-plane norms): the margin left under
    the 1e-4 bound."""
    import numpy as np

    path = REPO / "tests" / "golden" / f"{prefix}_{name}.npz"
    if not path.exists():
        return None
    with np.load(path, allow_pickle=False) as z:
        g = {k: z[k] for k in z.files}
    yh = y.detach().double().cpu().numpy()
    flat = yh.reshape(-1)
    sampled = float(np.abs(flat[g["sample_idx"]] - g["sample_val"].astype(np.float64)).max() / float(g["y_absmax"]))
    norms = np.sqrt((yh ** 2).sum(axis=(-2, -1)))
    norm_rel = float(np.abs(norms - g["y_plane_norm"]).max() / max(float(g["y_plane_norm"].max()), 1e-30))
    return {"max_abs_rel_sampled": sampled, "plane_norm_rel": norm_rel, "tol": 1e-4,
            "vs": f"tests/golden/{prefix}_{name}.npz (the reference's {ref} output)"}


class ClockSampler:
    """nvidia-smi sampling of SM clocks and throttle reasons while the GPU is loaded."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        try:
            import tempfile
            fd, self.path = tempfile.mkstemp(prefix="clocks_", suffix=".csv")
            os.close(fd)
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits", "-lms", "100",
                 "-i", str(self.gpu)], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()
        return False

    def summary(self) -> dict:
        out = {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
        if not self.path or not os.path.exists(self.path):
            return out
        rows = []
        for line in open(self.path):
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return out
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for _, _, flags in rows for i, f in enumerate(flags) if f.lower() == "active"})
        out.update(sm_mhz=statistics.median(r[0] for r in rows), sm_max_mhz=max(r[1] for r in rows),
                   reasons=reasons, samples=len(rows))
        return out


# ------------------------------------------------------------------------- our arm

def capture_graphs(device, fns) -> list:
    """One CUDA graph per callable; each is called with the capture stream's handle."""
    graphs = []
    cap = torch.cuda.Stream(device)
    cap.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(cap):
        for fn in fns:
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                fn(cap.cuda_stream)
            graphs.append(g)
    torch.cuda.current_stream(device).wait_stream(cap)
    return graphs


def run_spectral(name: str, steps: int, warmup: int, device, world: int, rank: int, *, with_e2e: bool,
                 with_breakdown: bool, sampler_gpu: int | None):
    import scx_data
    import spectral_conv_ext as ext
    import spectral_conv_ops as ops
    import scx_dist

    x_cpu, w1c, w2c, c = scx_data.make_spectral_case(name)
    B, Cin, Cout, H, W, m1, m2 = (c[k] for k in ("B", "Cin", "Cout", "H", "W", "m1", "m2"))
    w1 = torch.view_as_real(w1c.to(device)).contiguous()
    w2 = torch.view_as_real(w2c.to(device)).contiguous()
    per_set = 4 * B * H * W * (Cin + Cout)
    nsets = max(1, math.ceil(3 * L2_BYTES / per_set))
    xs = [x_cpu.to(device) for _ in range(nsets)]
    ys = [torch.empty(B, Cout, H, W, device=device) for _ in range(nsets)]
    ext.prepare(H, W, m1, m2)
    ws_bytes = ext._scx.lib.scx_spectral_conv2d_workspace_size(B, Cin, Cout, H, W, m1, m2)
    ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)
    lib = ext._scx.lib
    stream = torch.cuda.current_stream(device)
    sh = stream.cuda_stream

    def launch(i, stream_handle):
        s = i % nsets
        rc = lib.scx_spectral_conv2d_fwd(xs[s].data_ptr(), w1.data_ptr(), w2.data_ptr(), ys[s].data_ptr(), B, Cin,
                                         Cout, H, W, m1, m2, ws.data_ptr(), ws_bytes, stream_handle)
        if rc != 0:
            raise RuntimeError(f"scx_spectral_conv2d_fwd failed: {rc}")

    def barrier():
        if world > 1:
            torch.distributed.barrier()

    # CUDA graphs: n steps run as one graph of n forwards (three kernels each) over the input
    # sets in turn, so that every step keeps its programmatic overlap with the one before (a
    # graph launch per step, or per remainder step after whole rotations, adds its launch
    # latency to the step: at 64 x 64, 18 sets per rotation, that cost about 2.6 us per step)
    launch(0, sh)  # first use of the shape builds the twiddle tables outside any capture
    torch.cuda.synchronize(device)
    graphs = {}

    def run_steps(n):
        if n <= 0:
            return
        if n not in graphs:
            graphs[n] = capture_graphs(device, [lambda h: [launch(i, h) for i in range(n)]])[0]
        graphs[n].replay()

    for n in (warmup, steps, 4 * nsets, nsets):
        run_steps(n)  # captured (and run once) before the timed region
    torch.cuda.synchronize(device)

    run_steps(warmup)
    torch.cuda.synchronize(device)
    barrier()
    torch.cuda.synchronize(device)
    ev0 = torch.cuda.Event(enable_timing=True)
    ev1 = torch.cuda.Event(enable_timing=True)
    clocks = None
    sampler = ClockSampler(sampler_gpu) if sampler_gpu is not None else None
    if sampler:
        sampler.__enter__()
    ev0.record(stream)
    run_steps(steps)
    ev1.record(stream)
    torch.cuda.synchronize(device)
    t_ms = ev0.elapsed_time(ev1)
    if sampler:
        # keep the same load running for >= 1 s so that the 100 ms sampler sees it
        t_end = time.perf_counter() + 1.2
        while time.perf_counter() < t_end:
            run_steps(4 * nsets)
            torch.cuda.synchronize(device)
        sampler.__exit__()
        clocks = sampler.summary()
    # the same steps launched eagerly (one C-ABI call per step, no graph), for the latency
    # without graph replay
    run_steps(nsets)
    torch.cuda.synchronize(device)
    ev2 = torch.cuda.Event(enable_timing=True)
    ev3 = torch.cuda.Event(enable_timing=True)
    ev2.record(stream)
    for i in range(steps):
        launch(i, sh)
    ev3.record(stream)
    torch.cuda.synchronize(device)
    t_eager = scx_dist.max_over_ranks(ev2.elapsed_time(ev3), device)
    barrier()
    t_ms_max = scx_dist.max_over_ranks(t_ms, device)
    ms_per_step = t_ms_max / steps
    # 256-point grids run as a folding tensor-core forward, the mixing, four inverses and an
    # unfold; the per-kernel split below covers the three-kernel shapes
    n_launch = launches_per_forward(c)
    folded = n_launch != 3
    res = {"cfg": c, "ms_per_step": ms_per_step, "samples_per_s": world * B / (ms_per_step / 1e3),
           "ms_per_step_eager": t_eager / steps,
           "launches_per_step": n_launch, "clocks": clocks, "cuda_graph": True}
    if rank == 0:
        res["accuracy"] = fixture_error(name, ys[0])

    nbytes = spectral_bytes(c)
    peak, peak_kind = hbm_peak()
    res["roofline_fused_path"] = {
        "bound": "hbm", "achieved": nbytes["fused_path"] / (ms_per_step / 1e3) / 1e9, "peak": peak,
        "unit": "GB/s", "peak_kind": peak_kind, "bytes": nbytes["fused_path"]}
    res["roofline_fused_path"]["frac"] = res["roofline_fused_path"]["achieved"] / peak

    if with_breakdown and not folded:
        # per-kernel durations: each kernel replayed alone from a CUDA graph of nsets launches
        # (the inputs rotate as in the step), CUDA events around the replays
        ci = B * Cin * m1 * m2 * 2
        co = B * Cout * m1 * m2 * 2
        X1 = ws.view(torch.float32)[:ci]
        X2 = ws.view(torch.float32)[ci:2 * ci]
        Y1 = ws.view(torch.float32)[2 * ci:2 * ci + co]
        Y2 = ws.view(torch.float32)[2 * ci + co:2 * ci + 2 * co]

        def k_fwd(i, h):
            return lib.scx_rfft2_corners(xs[i % nsets].data_ptr(), X1.data_ptr(), X2.data_ptr(), B, Cin, H, W, m1,
                                         m2, h)

        def k_mix(i, h):
            return lib.scx_spectral_mul_dual(X1.data_ptr(), X2.data_ptr(), w1.data_ptr(), w2.data_ptr(),
                                             Y1.data_ptr(), Y2.data_ptr(), B, Cin, Cout, m1, m2, h)

        def k_inv(i, h):
            return lib.scx_irfft2_corners(Y1.data_ptr(), Y2.data_ptr(), ys[i % nsets].data_ptr(), B, Cout, H, W,
                                          m1, m2, h)

        kern = {}
        reps = max(10, steps)
        for kname, fn in (("dft_fwd", k_fwd), ("mix", k_mix), ("dft_inv", k_inv)):
            for i in range(nsets):  # warm, and check the status outside the capture
                rc = fn(i, sh)
                if rc != 0:
                    raise RuntimeError(f"{kname} failed: {rc}")
            torch.cuda.synchronize(device)
            g = capture_graphs(device, [lambda h: [fn(i, h) for i in range(nsets)]])[0]
            g.replay()
            e0 = torch.cuda.Event(enable_timing=True)
            e1 = torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize(device)
            kern[kname] = e0.elapsed_time(e1) / (reps * nsets)
            del g

        total = sum(kern.values())
        traffic = {}
        prof = REPO / "profiles" / "ncu_traffic.json"
        if prof.exists():
            try:
                traffic = json.loads(prof.read_text()).get(name, {})
            except Exception:
                traffic = {}
        res["kernels"] = {k: {"ms": v, "share": v / total, "bytes": nbytes[k],
                              "gbs": nbytes[k] / (v / 1e3) / 1e9, "frac": nbytes[k] / (v / 1e3) / 1e9 / peak,
                              "traffic": traffic.get(k)} for k, v in kern.items()}
        dom = max(kern, key=kern.get)
        achieved = nbytes[dom] / (kern[dom] / 1e3) / 1e9
        res["roofline"] = {"bound": "hbm", "kernel": dom, "achieved": achieved, "peak": peak, "unit": "GB/s",
                           "frac": achieved / peak, "peak_kind": peak_kind, "traffic": traffic.get(dom),
                           "bytes_per_launch": nbytes[dom], "ms_per_launch": kern[dom]}

    if with_e2e:
        # public host API: pinned host input in, host result out, copies inside the region
        x_host = x_cpu.pin_memory()
        w1p = w1c.to(device)
        w2p = w2c.to(device)
        n_e2e = max(3, min(steps, 20))
        # warm-up in the timed loop's pattern (the previous result alive during the next
        # call), so both page-locked result buffers exist before timing starts
        out = None
        for _ in range(3):
            out = ops.spectral_conv2d_supa(x_host, w1p, w2p, m1, m2, use_sufft="fused", to_cpu=True)
        torch.cuda.synchronize(device)
        barrier()
        t0 = time.perf_counter()
        for _ in range(n_e2e):
            out = ops.spectral_conv2d_supa(x_host, w1p, w2p, m1, m2, use_sufft="fused", to_cpu=True)
        torch.cuda.synchronize(device)
        t_e2e = (time.perf_counter() - t0) * 1e3 / n_e2e
        t_e2e = scx_dist.max_over_ranks(t_e2e, device)
        assert out.device.type == "cpu"
        res["e2e"] = {"value": world * B / (t_e2e / 1e3), "unit": "samples/s", "ms_per_step": t_e2e,
                      "h2d_bytes_per_step": x_host.numel() * 4, "d2h_bytes_per_step": out.numel() * 4,
                      "api": "spectral_conv_ops.spectral_conv2d_supa(to_cpu=True)"}
    return res


def run_strong(name: str, steps: int, warmup: int, device, world: int, rank: int) -> dict:
    """Strong scaling: the workload's whole batch (B=16 at 256x256, C64, m32) is split into
    contiguous shards over the ranks (16/8/4/2 items per GPU at N = 1/2/4/8); a step is the
    forward of this rank's shard and the gather of every shard into a preallocated
    [B, Cout, H, W] tensor on rank 0, as one CUDA graph: scx_dist.PipelinedGather, which runs
    the shard in sub-batches of two items and pushes each sub-batch's output to rank 0 by a peer
    copy while the next one is computed.  For comparison the line also times the forward of the whole
    shard followed by one push (``ms_per_step_push_after_forward``) and followed by the NCCL
    gather (``ms_per_step_nccl_gather``).  L2 is flushed (256 MiB write, not timed) before every
    step; each step has its own CUDA events on the launching stream, and the step time is the
    max over ranks.

    Rank 0 then runs the whole batch alone with the same protocol: its time is the one-GPU
    time the scaling efficiency is taken against, and its output is compared with the
    gathered one (sharded == single)."""
    import scx_data
    import scx_dist
    import spectral_conv_ext as ext

    x_cpu, w1c, w2c, c = scx_data.make_spectral_case(name)
    B, Cin, Cout, H, W, m1, m2 = (c[k] for k in ("B", "Cin", "Cout", "H", "W", "m1", "m2"))
    lib = ext._scx.lib
    w1 = torch.view_as_real(w1c.to(device)).contiguous()
    w2 = torch.view_as_real(w2c.to(device)).contiguous()
    ext.prepare(H, W, m1, m2)
    lo, hi = scx_dist.shard_range(B, world, rank)
    nb = hi - lo
    x_loc = x_cpu[lo:hi].contiguous().to(device)
    out_all = torch.empty(B, Cout, H, W, device=device) if rank == 0 else None
    # rank 0 computes its shard straight into its slice of the gathered output
    y_loc = out_all[lo:hi] if rank == 0 else torch.empty(nb, Cout, H, W, device=device)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    def make_forward(x, y, nbatch):
        ws_bytes = lib.scx_spectral_conv2d_workspace_size(nbatch, Cin, Cout, H, W, m1, m2)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=device)

        def fwd(h):
            rc = lib.scx_spectral_conv2d_fwd(x.data_ptr(), w1.data_ptr(), w2.data_ptr(), y.data_ptr(), nbatch, Cin,
                                             Cout, H, W, m1, m2, ws.data_ptr(), ws_bytes, h)
            if rc != 0:
                raise RuntimeError(f"scx_spectral_conv2d_fwd failed: {rc}")

        fwd(stream.cuda_stream)  # first use of the shape builds its tables outside the capture
        torch.cuda.synchronize(device)
        graph = capture_graphs(device, [fwd])[0]
        return graph, ws

    graph, ws_loc = make_forward(x_loc, y_loc, nb)

    def timed(step, n):
        evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(n)]
        for e0, e1 in evs:
            flush.zero_()
            e0.record(stream)
            step()
            e1.record(stream)
        torch.cuda.synchronize(device)
        return sum(e0.elapsed_time(e1) for e0, e1 in evs) / n

    peer = scx_dist.PeerGather(y_loc, out_all, B) if world > 1 else None

    def step_gather():
        graph.replay()
        if world > 1:
            peer.push(stream.cuda_stream)

    def step_nccl():
        graph.replay()
        if world > 1:
            scx_dist.gather_batch_into(y_loc, out_all, B)

    for _ in range(warmup):
        step_gather()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    t_fwd = scx_dist.max_over_ranks(timed(graph.replay, steps), device)
    t_nccl = None
    if world > 1:
        torch.distributed.barrier()
        for _ in range(warmup):
            step_nccl()
        t_nccl = scx_dist.max_over_ranks(timed(step_nccl, steps), device)
        torch.distributed.barrier()
    t_push_after = scx_dist.max_over_ranks(timed(step_gather, steps), device) if world > 1 else None
    t_step = t_push_after
    pipe = graph_pipe = None
    if world > 1:
        peer.sync()
        peer.close()  # the pipelined gather maps rank 0's output once more
        out_all_check = out_all.clone() if rank == 0 else None
        if rank == 0:
            out_all.fill_(float("nan"))  # the pipelined gather must fill every slot again
        torch.distributed.barrier()
        pipe = scx_dist.PipelinedGather(x_loc, y_loc, w1, w2, m1, m2, out_all, B)
        pipe.run(stream)  # outside any capture first
        torch.cuda.synchronize(device)
        graph_pipe = capture_graphs(device, [lambda h: pipe.run(torch.cuda.current_stream(device))])[0]
        for _ in range(warmup):
            graph_pipe.replay()
        torch.cuda.synchronize(device)
        torch.distributed.barrier()
        t_step = scx_dist.max_over_ranks(timed(graph_pipe.replay, steps), device)
        pipe.peer.sync()  # every push has landed before rank 0 reads the gathered output
        if rank == 0:
            # the sub-batch forwards may split the mixing's channel sum differently
            scale = max(out_all_check.abs().max().item(), 1e-30)
            pipelined_rel = (out_all - out_all_check).abs().max().item() / scale
    else:
        t_step = scx_dist.max_over_ranks(timed(step_gather, steps), device)
    res = {"workload": name, "batch_total": B, "batch_per_gpu": scx_dist.shard_sizes(B, world),
           "ms_per_step": t_step, "samples_per_s": B / (t_step / 1e3), "ms_forward_only": t_fwd,
           "gather_share": max(0.0, (t_step - t_fwd) / t_step) if world > 1 else 0.0,
           "gather": "peer copies into a preallocated tensor on rank 0 (CUDA IPC, copy engines over NVLink), "
                     "one per two-item sub-batch, each overlapping the next sub-batch's forward" if world > 1 else None,
           "ms_per_step_push_after_forward": t_push_after,
           "ms_per_step_nccl_gather": t_nccl,
           "launches_per_step": launches_per_forward(c), "cuda_graph": True, "scaling": "strong",
           "l2": "256 MiB flush between steps (not timed)"}
    if world > 1:
        torch.distributed.barrier()
    if rank == 0:
        if world > 1:
            x_all = x_cpu.to(device)
            y_all = torch.empty(B, Cout, H, W, device=device)
            graph1, ws1 = make_forward(x_all, y_all, B)
            for _ in range(warmup):
                graph1.replay()
            t_single = timed(graph1.replay, steps)
            del graph1, ws1
        else:
            y_all, t_single = out_all, t_step
        diff = (out_all - y_all).abs().max().item()
        scale = y_all.abs().max().item()
        res.update(ms_single_gpu=t_single, efficiency=t_single / (world * t_step),
                   # the mixing's tile shape (and so its split of the channel sum) depends on
                   # the batch size: equal up to that rounding, bitwise when the split agrees
                   sharded_equals_single=bool(diff <= 1e-5 * max(scale, 1e-30)),
                   sharded_bitwise_equal=bool(torch.equal(out_all, y_all)),
                   sharded_max_abs_rel_diff=diff / max(scale, 1e-30),
                   pipelined_vs_push_after_forward_rel=pipelined_rel if world > 1 else 0.0,
                   accuracy=fixture_error(name, out_all))
    if world > 1:
        torch.distributed.barrier()
        del graph_pipe
        pipe.close()
    del graph
    return res


def run_fno(steps: int, warmup: int, device, world: int, rank: int) -> dict:
    """FNO-NS forward, B=20 per GPU, [B,64,64,12] channels-last input, width 32, modes 12,
    4 layers, InstanceNorm layers; the whole forward is one libscx call replayed from a CUDA
    graph.  L2 is flushed (256 MiB write) between timed steps; each step is timed with its
    own CUDA events.  With N > 1 the step ends with the NCCL gather of all outputs to rank 0."""
    import fno_model
    import scx_data
    import scx_dist

    fw = scx_data.FNO_WORKLOAD
    torch.manual_seed(fw["init_seed"])
    model = fno_model.FNO2d(modes1=fw["modes"], modes2=fw["modes"], width=fw["width"], n_layers=fw["layers"],
                            in_channels=fw["frames"]).to(device)
    B = fw["B"]
    x = scx_data.fno_input(B, fw["seed"] + rank, H=fw["H"], W=fw["W"], frames=fw["frames"]).to(device)
    # the gathered [B * world] output lives on rank 0, which writes its own shard into it
    out_all = torch.empty(B * world, 1, fw["H"], fw["W"], device=device) if rank == 0 else None
    out = out_all[:B] if rank == 0 else torch.empty(B, 1, fw["H"], fw["W"], device=device)
    model.forward_device(x, channels_last=True, out=out)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        model.forward_device(x, channels_last=True, out=out)
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(graph):
        model.forward_device(x, channels_last=True, out=out)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)

    peer = scx_dist.PeerGather(out, out_all, B * world) if world > 1 else None

    def step():
        graph.replay()
        if world > 1:
            peer.push(stream.cuda_stream)

    for _ in range(warmup):
        step()
    torch.cuda.synchronize(device)
    if world > 1:
        torch.distributed.barrier()
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in evs:
        flush.zero_()
        e0.record(stream)
        step()
        e1.record(stream)
    torch.cuda.synchronize(device)
    t_ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    t_ms = scx_dist.max_over_ranks(t_ms, device)
    ms = t_ms / steps
    if world > 1:
        peer.sync()
        peer.close()
    del graph
    # rank 0's own shard has the seeds of the reference's fixture
    accuracy = fixture_error("fno_ns_b20_w32_64x64_m12_l4", out[:B], prefix="fno", ref="fno_ns/model.py") \
        if rank == 0 else None
    return {"ms_per_step": ms, "samples_per_s": world * B / (ms / 1e3), "batch_per_gpu": B, "accuracy": accuracy,
            # lift, then per layer forward DFT, mixing, inverse DFT and the fused skip +
            # instance norm + GELU (one cluster launch at 64x64), then the projection
            "launches_per_step": 2 + 4 * fw["layers"], "cuda_graph": True,
            "gather": "one peer copy per rank into a preallocated tensor on rank 0 (CUDA IPC, copy engines over "
                      "NVLink), inside the step" if world > 1 else None,
            "l2": "256 MiB flush between steps (not timed)"}


def run_backward(steps: int, warmup: int, device, world: int, rank: int) -> dict:
    """SpectralConv2d backward at the headline workload: grad_x and both weight gradients from
    grad_y and the forward's corner spectra (scx_spectral_conv2d_bwd: forward DFT of grad_y,
    two dual-corner mixings reading W^H and X^H in place, inverse DFT), replayed
    from a CUDA graph with a 256 MiB L2 flush between steps.  Algorithmic bytes: grad_y read,
    grad_x written, the weights read and their gradients written, the saved corners read."""
    import scx_data
    import scx_dist
    import spectral_conv_ext as ext

    x, w1, w2, c = scx_data.make_spectral_case(HEADLINE)
    B, Cin, Cout, H, W, m1, m2 = (c[k] for k in ("B", "Cin", "Cout", "H", "W", "m1", "m2"))
    w1d = torch.view_as_real(w1.to(device))
    w2d = torch.view_as_real(w2.to(device))
    _, xc = ext.spectral_conv2d_fwd_saved(x.to(device), w1d, w2d, m1, m2)
    gy = scx_data.gaussian((B, Cout, H, W), 77 + rank).to(device)
    ext.spectral_conv2d_bwd(gy, xc, w1d, w2d, m1, m2)
    torch.cuda.synchronize(device)
    graph = torch.cuda.CUDAGraph()
    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        ext.spectral_conv2d_bwd(gy, xc, w1d, w2d, m1, m2)
    torch.cuda.current_stream(device).wait_stream(side)
    with torch.cuda.graph(graph):
        grads = ext.spectral_conv2d_bwd(gy, xc, w1d, w2d, m1, m2)
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=device)
    stream = torch.cuda.current_stream(device)
    for _ in range(warmup):
        graph.replay()
    torch.cuda.synchronize(device)
    evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
    for e0, e1 in evs:
        flush.zero_()
        e0.record(stream)
        graph.replay()
        e1.record(stream)
    torch.cuda.synchronize(device)
    t_ms = sum(e0.elapsed_time(e1) for e0, e1 in evs)
    t_ms = scx_dist.max_over_ranks(t_ms, device)
    ms = t_ms / steps
    del graph, grads
    nm = m1 * m2
    nbytes = 4 * B * H * W * (Cin + Cout) + 2 * 2 * 8 * Cin * Cout * nm + 2 * 8 * B * Cin * nm
    peak, kind = hbm_peak()
    achieved = nbytes / (ms / 1e3) / 1e9
    return {"workload": HEADLINE, "ms_per_step": ms, "samples_per_s": world * B / (ms / 1e3),
            "launches_per_step": 4, "cuda_graph": True, "bytes_per_step": nbytes,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / peak, "peak_kind": kind},
            "l2": "256 MiB flush between steps (not timed)"}


def cpu_baseline(name: str, budget_s: float = 12.0) -> dict:
    """The reference's CPU recipe on the same workload, all host threads, bounded sample."""
    import scx_data
    from oracle import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    x, w1, w2, c = scx_data.make_spectral_case(name)
    oracle.spectral_conv2d_torch(x, w1, w2, c["m1"], c["m2"])  # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < 3 or (time.perf_counter() - t_start < budget_s and len(times) < 50):
        t0 = time.perf_counter()
        oracle.spectral_conv2d_torch(x, w1, w2, c["m1"], c["m2"])
        times.append(time.perf_counter() - t0)
        if time.perf_counter() - t_start > 4 * budget_s:
            break
    med = statistics.median(times)
    return {"value": c["B"] / med, "unit": "samples/s", "cores": torch.get_num_threads(), "kind": "port",
            "ms_per_step": med * 1e3,
            "sample": f"{len(times)} full forwards of {name} (B={c['B']}), median; torch.fft+einsum on CPU"}


def ours(args) -> None:
    import scx_dist

    rank, local_rank, world = scx_dist.env_rank()
    if world != args.gpus:
        if world == 1 and args.gpus > 1:
            raise SystemExit("--gpus N>1 needs torchrun (one process per GPU)")
    if not torch.cuda.is_available():
        raise SystemExit("bench.py needs a CUDA device")
    torch.cuda.set_device(local_rank)
    device = torch.device("cuda", local_rank)
    if world > 1:
        # NCCL's version banner would land on stdout ahead of the one JSON line
        if os.environ.get("NCCL_DEBUG", "VERSION").upper() == "VERSION":
            os.environ["NCCL_DEBUG"] = "WARN"
        scx_dist.init("nccl", timeout_s=300, device=device)
    warmup = max(3, args.warmup)
    res = run_spectral(args.workload, args.steps, warmup, device, world, rank, with_e2e=True,
                       with_breakdown=True, sampler_gpu=local_rank if rank == 0 else None)
    extras = {}
    wanted = {"64", "256", "irr", "c3s", "fno", "bwd"} if args.extras == "all" else set(args.extras.split(","))
    if not args.no_extras:
        for wname in EXTRA_WORKLOADS:
            if wname == args.workload or wname.split("_")[3].split("x")[0] not in wanted:
                continue
            r = run_spectral(wname, max(10, args.steps // 2), warmup, device, world, rank, with_e2e=False,
                             with_breakdown=True, sampler_gpu=None)
            extras[wname] = {"ms_per_step": r["ms_per_step"], "samples_per_s": r["samples_per_s"],
                             "ms_per_step_eager": r["ms_per_step_eager"],
                             "roofline_fused_path_frac": r["roofline_fused_path"]["frac"],
                             "launches_per_step": r["launches_per_step"], "cuda_graph": True,
                             "accuracy": r.get("accuracy")}
            if "roofline" in r:
                extras[wname].update(dominant_kernel=r["roofline"]["kernel"],
                                     dominant_kernel_frac=r["roofline"]["frac"],
                                     kernels_ms={k: v["ms"] for k, v in r["kernels"].items()})
        if "irr" in wanted:
            for wname in IRREGULAR_WORKLOADS:
                r = run_spectral(wname, max(10, args.steps // 2), warmup, device, world, rank, with_e2e=False,
                                 with_breakdown=True, sampler_gpu=None)
                extras[wname] = {"ms_per_step": r["ms_per_step"], "samples_per_s": r["samples_per_s"],
                                 "ms_per_step_eager": r["ms_per_step_eager"],
                                 "roofline_fused_path_frac": r["roofline_fused_path"]["frac"],
                                 "launches_per_step": r["launches_per_step"], "cuda_graph": True,
                                 "accuracy": r.get("accuracy")}
                if "roofline" in r:
                    extras[wname].update(dominant_kernel=r["roofline"]["kernel"],
                                         dominant_kernel_frac=r["roofline"]["frac"],
                                         kernels_ms={k: v["ms"] for k, v in r["kernels"].items()})
        if "c3s" in wanted:
            extras["c3_strong_" + STRONG_WORKLOAD] = run_strong(STRONG_WORKLOAD, max(10, args.steps // 2), warmup,
                                                                device, world, rank)
        if "fno" in wanted:
            extras["fno_ns_b20_w32_64x64_m12_l4"] = run_fno(max(10, args.steps // 2), warmup, device, world, rank)
        if "bwd" in wanted:
            extras["spectral_bwd_b20_c32_128x128_m16"] = run_backward(max(10, args.steps // 2), warmup, device,
                                                                      world, rank)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.workload)
    if rank == 0:
        c = res["cfg"]
        line = {
            "metric": "SpectralConv2d fwd samples/s (per-GPU B20, Cin=Cout=32, 128x128, modes 16, GRF input)"
            if args.workload == HEADLINE else f"SpectralConv2d fwd samples/s ({args.workload})",
            "value": res["samples_per_s"], "unit": "samples/s", "n_gpus": world, "steps": args.steps,
            "warmup": warmup, "ms_per_step": res["ms_per_step"], "ms_per_step_eager": res["ms_per_step_eager"],
            "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded Gaussian random field)",
            "config": {"workload": args.workload, "batch_per_gpu": c["B"], "global_batch": c["B"] * world,
                       "channels_in": c["Cin"], "channels_out": c["Cout"], "height": c["H"], "width": c["W"],
                       "modes1": c["m1"], "modes2": c["m2"], "parallelism": f"batch-shard x{world}",
                       "l2": "inputs rotate over buffer sets totalling >= 3x L2 between steps",
                       "launch": "CUDA graphs of whole rotations over the buffer sets (three kernels per forward)"},
            "roofline": res.get("roofline"), "roofline_fused_path": res["roofline_fused_path"],
            "kernels": res.get("kernels"), "e2e": res.get("e2e"), "cpu_baseline": cpu,
            "accuracy": res.get("accuracy"),
            "clocks": res["clocks"], "gpu_launches": res["launches_per_step"] * args.steps,
            "workloads": extras,
        }
        emit(line)
    if world > 1:
        torch.distributed.barrier()
        torch.distributed.destroy_process_group()


def reference(args) -> None:
    import scx_dist

    rank, _, world = scx_dist.env_rank()
    if rank != 0:
        return
    import scx_data
    from oracle import oracle

    torch.set_num_threads(os.cpu_count() or 1)
    x, w1, w2, c = scx_data.make_spectral_case(args.workload)
    warmup = max(3, args.warmup)
    # bound the run to a few minutes: one full forward per step when it is short enough,
    # otherwise a batch slice of the same workload
    t0 = time.perf_counter()
    oracle.spectral_conv2d_torch(x, w1, w2, c["m1"], c["m2"])
    t_one = time.perf_counter() - t0
    budget = 150.0
    nb = c["B"]
    if t_one * (warmup + args.steps) > budget:
        nb = max(1, int(c["B"] * budget / (t_one * (warmup + args.steps))))
    xs = x[:nb].contiguous()
    for _ in range(warmup):
        oracle.spectral_conv2d_torch(xs, w1, w2, c["m1"], c["m2"])
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.spectral_conv2d_torch(xs, w1, w2, c["m1"], c["m2"])
    dt = (time.perf_counter() - t0) / args.steps
    value = nb / dt
    line = {
        "impl": "reference", "metric": "SpectralConv2d fwd samples/s (per-GPU B20, Cin=Cout=32, 128x128, modes 16,"
        " GRF input)" if args.workload == HEADLINE else f"SpectralConv2d fwd samples/s ({args.workload})",
        "value": value, "unit": "samples/s", "n_gpus": world, "steps": args.steps, "warmup": warmup,
        "ms_per_step": dt * 1e3, "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded Gaussian random field)",
        "config": {"workload": args.workload, "batch_per_step": nb, "channels_in": c["Cin"],
                   "channels_out": c["Cout"], "height": c["H"], "width": c["W"], "modes1": c["m1"],
                   "modes2": c["m2"]},
        "cpu_baseline": {"value": value, "unit": "samples/s", "cores": torch.get_num_threads(), "kind": "port",
                         "sample": f"{args.steps} forwards of {nb} batch items; the reference's torch.fft + "
                                   "einsum recipe (reference_pytorch.py) restated, on the host CPU"},
        "e2e": {"value": value, "unit": "samples/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    emit(line)


# The JSON result line goes to the process's original stdout; file descriptor 1 itself is
# pointed at stderr, so that banners printed by native libraries (NCCL's version line, for
# one) cannot land in front of it.
_RESULT_OUT = None


def emit(line: dict) -> None:
    out = _RESULT_OUT if _RESULT_OUT is not None else sys.stdout
    print(json.dumps(line), file=out, flush=True)


def main() -> None:
    global _RESULT_OUT
    sys.stdout.flush()
    _RESULT_OUT = os.fdopen(os.dup(1), "w")
    os.dup2(2, 1)
    args = parse_args()
    if args.impl == "reference":
        reference(args)
    else:
        ours(args)


if __name__ == "__main__":
    main()
