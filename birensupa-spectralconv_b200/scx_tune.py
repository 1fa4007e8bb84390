"""Per-shape kernel-variant table: the B200 counterpart of the reference's tuning sweep
(spectral_conv_combo/tune.py:154-261) and its ``_AUTO_TUNE_TABLE``
(spectral_conv_combo/spectral_conv_ops.py:45-63).

The reference sweeps {v1, fused} x buffer sizes x a ``fused_block`` knob that no kernel reads,
writes ``tune_results.json`` and never reads it back.  Here the sweep is over the kernels that
really differ for a shape, each timed on the device, and the table is persisted and reloaded:

* truncated DFTs, per (H, W, m1, m2): FFMA direct DFT, tensor-core kernels, or the folded
  tensor-core path (``scx_dft_variants`` says which apply);
* mixing, per (corners, B, Cin, Cout, m1*m2): each TMA-ring tile shape, the per-thread kernel
  or the tensor-core (3xTF32) kernel.

Every candidate is timed as the whole fused forward (CUDA graph of rotating input sets larger
than L2, CUDA events) and its output is checked against the library's default choice before it
can win.  ``load()`` applies a saved table through ``scx_set_dft_variant`` /
``scx_set_mix_variant``; ``spectral_conv_ops`` calls it at import when ``SCX_TUNE_TABLE``
names a file (or the package's ``tune_table.json`` exists).

    python birensupa-spectralconv_b200/scx_tune.py --workloads spectral_b20_c32_64x64_m12 --out table.json
"""

from __future__ import annotations

import argparse
import json
import math
import os
import sys
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
if str(PKG_DIR) not in sys.path:
    sys.path.insert(0, str(PKG_DIR))

import _scx  # noqa: E402

TABLE_ENV = "SCX_TUNE_TABLE"
DFT_NAMES = {0: "auto", 1: "ffma", 2: "tensor", 3: "folded"}
DFT_CODES = {v: k for k, v in DFT_NAMES.items()}
MIX_SMEM = 8
MIX_TC = 9  # the tcgen05 3xTF32 kernel (wide channel counts; other shapes fall back to the default)
MIX_RING_SHAPES = 8  # tile shapes 0..7 of the TMA-ring mixing kernel
L2_BYTES = 126 * 1024 * 1024
TOL = 1e-5  # a variant may differ from the default choice only by rounding
MARGIN = 0.02  # a variant replaces the current best only when it is faster by more than this


def default_path() -> Path:
    env = os.environ.get(TABLE_ENV)
    return Path(env) if env else PKG_DIR / "tune_table.json"


def empty_table() -> dict:
    return {"version": 1, "dft": [], "mix": []}


def apply(table: dict) -> int:
    """Sets every entry of ``table`` in the library; returns how many were applied.  Entries
    whose variant does not apply to their shape are skipped (the library refuses them)."""
    n = 0
    for e in table.get("dft", []):
        code = DFT_CODES.get(e["variant"]) if isinstance(e["variant"], str) else int(e["variant"])
        if code is not None and _scx.lib.scx_set_dft_variant(e["H"], e["W"], e["m1"], e["m2"], code) == 0:
            n += 1
    for e in table.get("mix", []):
        if _scx.lib.scx_set_mix_variant(e["corners"], e["B"], e["Cin"], e["Cout"], e["modes"], int(e["variant"])) == 0:
            n += 1
    return n


def load(path: str | os.PathLike | None = None) -> int:
    """Reads a saved table (default: ``default_path()``) and applies it; 0 if there is none."""
    p = Path(path) if path is not None else default_path()
    if not p.exists():
        return 0
    return apply(json.loads(p.read_text()))


def save(table: dict, path: str | os.PathLike | None = None) -> Path:
    p = Path(path) if path is not None else default_path()
    p.write_text(json.dumps(table, indent=1, sort_keys=True) + "\n")
    return p


def merge(table: dict, entry: dict, kind: str) -> None:
    """Adds ``entry`` to ``table[kind]``, replacing an entry for the same shape."""
    keys = ("H", "W", "m1", "m2") if kind == "dft" else ("corners", "B", "Cin", "Cout", "modes")
    table[kind] = [e for e in table[kind] if any(e[k] != entry[k] for k in keys)] + [entry]


class _Forward:
    """The fused forward of one shape on rotating input sets, timed from a CUDA graph."""

    def __init__(self, x_cpu, w1, w2, c, device):
        self.c = c
        B, Cin, Cout, H, W = (c[k] for k in ("B", "Cin", "Cout", "H", "W"))
        per_set = 4 * B * H * W * (Cin + Cout)
        self.nsets = max(1, math.ceil(2 * L2_BYTES / per_set))
        self.xs = [x_cpu.to(device) for _ in range(self.nsets)]
        self.ys = [torch.empty(B, Cout, H, W, device=device) for _ in range(self.nsets)]
        self.w1 = torch.view_as_real(w1.to(device)).contiguous()
        self.w2 = torch.view_as_real(w2.to(device)).contiguous()
        self.ws_bytes = _scx.lib.scx_spectral_conv2d_workspace_size(B, Cin, Cout, H, W, c["m1"], c["m2"])
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=device)
        self.device = device

    def launch(self, i, stream):
        c = self.c
        rc = _scx.lib.scx_spectral_conv2d_fwd(self.xs[i].data_ptr(), self.w1.data_ptr(), self.w2.data_ptr(),
                                              self.ys[i].data_ptr(), c["B"], c["Cin"], c["Cout"], c["H"], c["W"],
                                              c["m1"], c["m2"], self.ws.data_ptr(), self.ws_bytes, stream)
        _scx.check(rc, "scx_spectral_conv2d_fwd")

    def time_ms(self, reps: int = 20) -> float:
        dev = self.device
        h = torch.cuda.current_stream(dev).cuda_stream
        for i in range(self.nsets):  # first use of a variant builds its tables outside the capture
            self.launch(i, h)
        torch.cuda.synchronize(dev)
        side = torch.cuda.Stream(dev)
        side.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(side):
            with torch.cuda.graph(g, stream=side):
                for i in range(self.nsets):
                    self.launch(i, side.cuda_stream)
        torch.cuda.current_stream(dev).wait_stream(side)
        g.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(reps):
            g.replay()
        e1.record()
        torch.cuda.synchronize(dev)
        del g
        return e0.elapsed_time(e1) / (reps * self.nsets)

    def output(self) -> torch.Tensor:
        return self.ys[0].clone()


def _close(ref: torch.Tensor, got: torch.Tensor) -> bool:
    scale = ref.abs().max().item()
    return bool(torch.isfinite(got).all()) and (got - ref).abs().max().item() <= TOL * max(scale, 1e-30)


def tune_spectral(x_cpu, w1, w2, c: dict, device, reps: int = 20, log=None) -> tuple[dict, dict, dict]:
    """Measures the variants of one SpectralConv2d shape.  Returns (dft entry, mix entry,
    times) with the fastest DFT variant (mixing at the library's choice) and then the fastest
    mixing variant (with that DFT variant); each candidate's output must match the default's,
    and it must beat the best so far by more than MARGIN (a tile shape that does not fit the
    shape falls back to the default and so times the same)."""
    lib = _scx.lib
    H, W, m1, m2 = c["H"], c["W"], c["m1"], c["m2"]
    mix_key = (2, c["B"], c["Cin"], c["Cout"], m1 * m2)
    lib.scx_set_dft_variant(H, W, m1, m2, 0)
    lib.scx_set_mix_variant(*mix_key, -1)
    fwd = _Forward(x_cpu, w1, w2, c, device)
    times = {"default": fwd.time_ms(reps)}
    ref = fwd.output()
    mask = lib.scx_dft_variants(H, W, m1, m2)
    best_dft, best_t = 0, times["default"]
    for code in (1, 2, 3):
        if not mask & (1 << code):
            continue
        lib.scx_set_dft_variant(H, W, m1, m2, code)
        t = fwd.time_ms(reps)
        ok = _close(ref, fwd.output())
        times[f"dft_{DFT_NAMES[code]}"] = t if ok else None
        if log:
            log(f"  dft {DFT_NAMES[code]:7s} {t * 1e3:8.1f} us{'' if ok else '  (rejected: output differs)'}")
        if ok and t < best_t * (1 - MARGIN):
            best_dft, best_t = code, t
    lib.scx_set_dft_variant(H, W, m1, m2, best_dft)
    best_mix = -1
    for v in list(range(MIX_RING_SHAPES)) + [MIX_SMEM, MIX_TC]:
        lib.scx_set_mix_variant(*mix_key, v)
        t = fwd.time_ms(reps)
        ok = _close(ref, fwd.output())
        times[f"mix_{v}"] = t if ok else None
        if log:
            log(f"  mix {v:7d} {t * 1e3:8.1f} us{'' if ok else '  (rejected: output differs)'}")
        if ok and t < best_t * (1 - MARGIN):
            best_mix, best_t = v, t
    lib.scx_set_mix_variant(*mix_key, best_mix)
    dft_entry = {"H": H, "W": W, "m1": m1, "m2": m2, "variant": DFT_NAMES[best_dft], "ms": best_t,
                 "ms_default": times["default"]}
    mix_entry = {"corners": 2, "B": c["B"], "Cin": c["Cin"], "Cout": c["Cout"], "modes": m1 * m2,
                 "variant": best_mix, "ms": best_t, "ms_default": times["default"]}
    return dft_entry, mix_entry, times


def main(argv=None) -> None:
    import scx_data

    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--workloads", default=",".join(scx_data.SPECTRAL_WORKLOADS),
                    help="comma list of scx_data.SPECTRAL_WORKLOADS names")
    ap.add_argument("--out", default=None, help=f"table file (default: ${TABLE_ENV} or the package's tune_table.json)")
    ap.add_argument("--reps", type=int, default=20)
    args = ap.parse_args(argv)
    device = torch.device("cuda", torch.cuda.current_device())
    out = Path(args.out) if args.out else default_path()
    table = json.loads(out.read_text()) if out.exists() else empty_table()
    table["device"] = torch.cuda.get_device_name(device)
    for name in args.workloads.split(","):
        x, w1, w2, c = scx_data.make_spectral_case(name)
        print(f"{name}:", flush=True)
        d, m, _ = tune_spectral(x, w1, w2, c, device, args.reps, log=lambda s: print(s, flush=True))
        merge(table, d, "dft")
        merge(table, m, "mix")
        print(f"  -> dft {d['variant']}, mix {m['variant']}: {m['ms'] * 1e3:.1f} us "
              f"(default {m['ms_default'] * 1e3:.1f} us)", flush=True)
    print(f"wrote {save(table, out)}")


if __name__ == "__main__":
    main()
