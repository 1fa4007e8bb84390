"""Generates the golden fixtures in this folder by running the REFERENCE implementation.

Run once where a checkout of the reference is available, passing its root (or setting
``SCX_REFERENCE_ROOT``); the fixtures are committed and the tests never read the reference:

    python tests/golden/make_golden.py --reference <reference checkout>

What runs (all on the CPU, fp32, exactly the reference's code):
* ``spectral_conv/reference_pytorch.py: SpectralConv2d`` on
  - the five cases of ``spectral_conv_combo/test_accuracy.py:61-65`` (their seed recipe),
  - the nine shapes of ``spectral_conv_combo/test_irregular_shapes.py:22-32``,
  - the named benchmark workloads (seeded synthetic inputs);
* ``spectral_conv_combo/reference_pytorch.py: spectral_conv3d`` on the two cases of
  ``spectral_conv_combo/test_3d_accuracy.py:69-72``, and ``official_baseline.py:
  SpectralConv3d`` (four corners) on seeded cases (``--only conv3d`` makes just these);
* ``fno_ns/model.py: FNO2d.forward(x, use_supa=False)`` (imported with a stub for its
  SUPA-only ``spectral_conv_ops`` import) at width 32, modes 12, 4 layers, on the seeded
  Navier-Stokes-like input.

Small outputs are stored whole; large ones as per-plane sums / norms plus 4096 sampled
values (``sample_idx`` into the flattened output), with input checksums so a test can
confirm it regenerated the same inputs.
"""

from __future__ import annotations

import argparse
import os
import importlib.util
import sys
import types
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO / "birensupa-spectralconv_b200"))
import scx_data  # noqa: E402

FULL_LIMIT = 1 << 16  # store inputs and outputs with at most this many elements whole
N_SAMPLES = 4096


def _load_module(path: Path, name: str):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _summary(y: torch.Tensor, seed: int) -> dict:
    y = y.detach().to(torch.float64)
    flat = y.reshape(-1)
    rng = np.random.default_rng(seed)
    idx = np.sort(rng.choice(flat.numel(), size=min(N_SAMPLES, flat.numel()), replace=False))
    out = {
        "y_plane_sum": y.sum(dim=(-2, -1)).numpy(),
        "y_plane_norm": y.pow(2).sum(dim=(-2, -1)).sqrt().numpy(),
        "y_norm": np.float64(flat.norm().item()),
        "y_absmax": np.float64(flat.abs().max().item()),
        "sample_idx": idx.astype(np.int64),
        "sample_val": flat[torch.from_numpy(idx)].numpy().astype(np.float32),
    }
    if flat.numel() <= FULL_LIMIT:
        out["y"] = y.to(torch.float32).numpy()
    return out


def _input_sums(x, w1, w2) -> dict:
    return {
        "x_sum": np.float64(x.double().sum().item()),
        "x_sumsq": np.float64(x.double().pow(2).sum().item()),
        "w1_sum": np.complex128(w1.to(torch.complex128).sum().item()),
        "w2_sum": np.complex128(w2.to(torch.complex128).sum().item()),
    }


def spectral_fixture(ref_mod, name, recipe, B, Cin, Cout, H, W, m1, m2, x, w1, w2, seed):
    layer = ref_mod.SpectralConv2d(Cin, Cout, m1, m2)
    with torch.no_grad():
        layer.weights1.copy_(w1)
        layer.weights2.copy_(w2)
        y = layer(x)
    data = dict(name=name, recipe=recipe, B=B, Cin=Cin, Cout=Cout, H=H, W=W, m1=m1, m2=m2, seed=seed)
    data.update(_input_sums(x, w1, w2))
    data.update(_summary(y, seed + 12345))
    if x.numel() <= FULL_LIMIT:
        data.update(x=x.numpy(), w1=w1.numpy(), w2=w2.numpy())
    np.savez_compressed(HERE / f"spectral_{name}.npz", **data)
    print(f"spectral_{name}: y{tuple(y.shape)} |y|={float(y.norm()):.6g}")


def conv3d_fixtures(ref: Path) -> None:
    """spectral_conv_combo/reference_pytorch.py: spectral_conv3d on the two cases of
    spectral_conv_combo/test_3d_accuracy.py:69-72, with that test's input recipe
    (make_random_weights of the same file for the weights); stored whole."""
    mod = _load_module(ref / "spectral_conv_combo" / "reference_pytorch.py", "reference_pytorch_combo")
    for (name, B, Cin, Cout, D, H, W, modes, seed) in scx_data.REFERENCE_3D_CASES:
        x, w = scx_data.reference_3d_case(B, Cin, Cout, D, H, W, modes, seed)
        w_ref = mod.make_random_weights(Cin, Cout, modes[0], modes[1] * modes[2], seed + 1)
        assert torch.equal(w_ref.reshape(w.shape), w)
        y = mod.spectral_conv3d(x, w, *modes)
        np.savez_compressed(HERE / f"conv3d_{name}.npz", name=name, B=B, Cin=Cin, Cout=Cout, D=D, H=H, W=W,
                            modes=np.array(modes), seed=seed, x=x.numpy(), w=w.numpy(),
                            y=y.detach().numpy())
        print(f"conv3d {name}: y{tuple(y.shape)} |y|={float(y.norm()):.6g}")


def official3d_fixtures(ref: Path) -> None:
    """spectral_conv_combo/official_baseline.py: SpectralConv3d (four corners) on seeded
    inputs, initialised under torch.manual_seed; weights, inputs and outputs stored whole."""
    mod = _load_module(ref / "spectral_conv_combo" / "official_baseline.py", "official_baseline_combo")
    for (name, B, Cin, Cout, D, H, W, modes, seed) in scx_data.OFFICIAL_3D_CASES:
        torch.manual_seed(seed)
        layer = mod.SpectralConv3d(Cin, Cout, *modes)
        x = torch.randn(B, Cin, D, H, W, generator=torch.Generator().manual_seed(seed + 1))
        with torch.no_grad():
            y = layer(x)
        ws = {f"w{i}": getattr(layer, f"weights{i}").detach().numpy() for i in range(1, 5)}
        np.savez_compressed(HERE / f"conv3d_{name}.npz", name=name, B=B, Cin=Cin, Cout=Cout, D=D, H=H, W=W,
                            modes=np.array(modes), seed=seed, x=x.numpy(), y=y.numpy(), **ws)
        print(f"official 3-D {name}: y{tuple(y.shape)} |y|={float(y.norm()):.6g}")


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("SCX_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $SCX_REFERENCE_ROOT)")
    ap.add_argument("--only", choices=["all", "conv3d"], default="all")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference <reference checkout> or set SCX_REFERENCE_ROOT")
    ref = Path(args.reference)
    torch.set_num_threads(8)
    conv3d_fixtures(ref)
    official3d_fixtures(ref)
    if args.only == "conv3d":
        return
    ref_mod = _load_module(ref / "spectral_conv" / "reference_pytorch.py", "reference_pytorch")

    for (name, B, Cin, Cout, H, W, m1, m2, seed) in scx_data.REFERENCE_ACCURACY_CASES:
        x, w1, w2 = scx_data.reference_accuracy_case(B, Cin, Cout, H, W, m1, m2, seed)
        # same draws as the reference's own module construction
        torch.manual_seed(seed)
        probe = ref_mod.SpectralConv2d(Cin, Cout, m1, m2)
        assert torch.equal(probe.weights1.detach(), w1) and torch.equal(probe.weights2.detach(), w2)
        spectral_fixture(ref_mod, f"refacc_{name}", "reference_accuracy", B, Cin, Cout, H, W, m1, m2,
                         x, w1, w2, seed)

    for (B, Cin, H, W) in scx_data.REFERENCE_IRREGULAR_SHAPES:
        x, w1, w2, M = scx_data.reference_irregular_case(B, Cin, H, W)
        spectral_fixture(ref_mod, f"refirr_{B}x{Cin}x{H}x{W}", "reference_irregular", B, Cin, 64, H, W,
                         M, M, x, w1, w2, 0)

    for name in scx_data.SPECTRAL_WORKLOADS:
        x, w1, w2, c = scx_data.make_spectral_case(name)
        spectral_fixture(ref_mod, name, "workload", c["B"], c["Cin"], c["Cout"], c["H"], c["W"], c["m1"],
                         c["m2"], x, w1, w2, c["seed"])

    # FNO-2d (fno_ns/model.py) with its SUPA import stubbed out.
    stub = types.ModuleType("spectral_conv_ops")
    stub.spectral_conv2d_supa = None
    sys.modules["spectral_conv_ops"] = stub
    model_mod = _load_module(ref / "fno_ns" / "model.py", "fno_reference_model")
    fw = scx_data.FNO_WORKLOAD
    torch.manual_seed(fw["init_seed"])
    model = model_mod.FNO2d(modes1=fw["modes"], modes2=fw["modes"], width=fw["width"],
                            n_layers=fw["layers"], in_channels=fw["frames"])
    model.eval()
    x_cl = scx_data.fno_input(fw["B"], fw["seed"], H=fw["H"], W=fw["W"], frames=fw["frames"])
    x = x_cl[..., : fw["frames"]].permute(0, 3, 1, 2).contiguous()
    with torch.no_grad():
        y = model(x, use_supa=False)
    data = dict(name=fw["name"], B=fw["B"], H=fw["H"], W=fw["W"], frames=fw["frames"],
                width=fw["width"], modes=fw["modes"], layers=fw["layers"], seed=fw["seed"],
                init_seed=fw["init_seed"])
    data["x_sum"] = np.float64(x_cl.double().sum().item())
    data["x_sumsq"] = np.float64(x_cl.double().pow(2).sum().item())
    names = []
    sums = []
    for k, v in model.state_dict().items():
        names.append(k)
        vv = v.detach()
        sums.append(complex(vv.to(torch.complex128).sum().item()) if vv.is_complex()
                    else complex(vv.double().sum().item(), 0.0))
    data["param_names"] = np.array(names)
    data["param_sums"] = np.array(sums, dtype=np.complex128)
    data.update(_summary(y, 777))
    np.savez_compressed(HERE / f"fno_{fw['name']}.npz", **data)
    print(f"fno: y{tuple(y.shape)} |y|={float(y.norm()):.6g}")


if __name__ == "__main__":
    main()
