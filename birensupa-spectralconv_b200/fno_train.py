"""FNO-NS training on the device: the loop of fno_ns/train_official.py:56-154 with the data
generated, and the forward and backward run, on a CUDA device.

Reference recipe kept: FNO2d(width 32, 4 layers, 10 input frames), Adam(lr 2e-4, weight decay
1e-4), CosineAnnealingLR over the epochs (T_max = max(epochs, 3)), batch 16, the loss
||pred - y|| / ||y|| per batch, the test score as the mean per-sample relative L2
(``relative_l2``, train_official.py:41-44), and the best-test-L2 checkpoint.  Differences:

* the data are ``scx_data.fno_pairs_device`` (the pseudo-spectral NS generator on the device,
  transforms on the library's kernels) instead of the reference's host-side NS-like cache;
* the training forward is ``FNO2d.forward_autograd`` (spectral convolutions on the library's
  forward and backward kernels) and evaluation runs the fused one-call forward
  (``FNO2d.forward_device``), instead of the reference's CPU torch path (``use_supa=False``);
* batches are drawn from a seeded permutation on the device, not a host DataLoader.

    python birensupa-spectralconv_b200/fno_train.py --epochs 5 --n-train 256 --n-test 64
"""

from __future__ import annotations

import argparse
import json
import sys
import time
from pathlib import Path

import torch

PKG_DIR = Path(__file__).resolve().parent
if str(PKG_DIR) not in sys.path:
    sys.path.insert(0, str(PKG_DIR))

import fno_model  # noqa: E402
import scx_data  # noqa: E402


def relative_l2(pred: torch.Tensor, target: torch.Tensor) -> float:
    """Mean over samples of ||pred - target|| / ||target|| per field
    (fno_ns/train_official.py:41-44)."""
    diff = torch.norm(pred - target, dim=(-2, -1))
    ref = torch.norm(target, dim=(-2, -1)).clamp_min(1.0e-12)
    return float((diff / ref).mean().item())


def evaluate(model: fno_model.FNO2d, x: torch.Tensor, y: torch.Tensor, batch_size: int) -> float:
    """Test score with the fused device forward, batch by batch (train_official.py:47-53)."""
    model.eval()
    scores = []
    with torch.no_grad():
        for i in range(0, x.shape[0], batch_size):
            scores.append(relative_l2(model.forward_device(x[i:i + batch_size]), y[i:i + batch_size]))
    return sum(scores) / max(len(scores), 1)


def train(model: fno_model.FNO2d, x_train, y_train, x_test, y_test, *, epochs: int, batch_size: int = 16,
          lr: float = 2.0e-4, weight_decay: float = 1.0e-4, seed: int = 0, scheduler: bool = True,
          checkpoint: str | None = None, log=print) -> dict:
    """Trains ``model`` (on the data's device) and returns a summary with the per-epoch losses."""
    device = x_train.device
    g = torch.Generator(device=device)
    g.manual_seed(seed)
    optim = torch.optim.Adam(model.parameters(), lr=lr, weight_decay=weight_decay)
    sched = torch.optim.lr_scheduler.CosineAnnealingLR(optim, T_max=max(epochs, 3)) if scheduler else None
    n = x_train.shape[0]
    history, best_l2, step = [], float("inf"), 0
    t0 = time.time()
    for epoch in range(epochs):
        model.train()
        order = torch.randperm(n, generator=g, device=device)
        loss_sum, count = 0.0, 0
        for i in range(0, n, batch_size):
            idx = order[i:i + batch_size]
            x, y = x_train[idx], y_train[idx]
            optim.zero_grad()
            pred = model.forward_autograd(x)
            loss = torch.norm(pred - y) / torch.norm(y).clamp_min(1e-12)
            loss.backward()
            optim.step()
            loss_sum += float(loss.item())
            count += 1
            step += 1
        if sched is not None:
            sched.step()
        train_l2 = loss_sum / max(count, 1)
        test_l2 = evaluate(model, x_test, y_test, batch_size)
        improved = test_l2 < best_l2
        if improved:
            best_l2 = test_l2
            if checkpoint:
                torch.save({"model": model.state_dict(), "test_l2": test_l2, "step": step, "epoch": epoch + 1},
                           checkpoint)
        history.append({"epoch": epoch + 1, "step": step, "train_l2": train_l2, "test_l2": test_l2,
                        "lr": optim.param_groups[0]["lr"]})
        log(f"step {step:5d} | epoch {epoch + 1:3d} | train_l2={train_l2:.6f} | test_l2={test_l2:.6f} | "
            f"best_l2={best_l2:.6f}{'  *best*' if improved else ''}")
    torch.cuda.synchronize(device)
    return {"epochs": epochs, "steps": step, "best_test_l2": best_l2, "history": history,
            "elapsed_s": time.time() - t0, "n_train": n, "n_test": int(x_test.shape[0]), "batch_size": batch_size}


def main(argv=None) -> None:
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--epochs", type=int, default=10)
    ap.add_argument("--n-train", type=int, default=1000)
    ap.add_argument("--n-test", type=int, default=128)
    ap.add_argument("--batch-size", type=int, default=16)
    ap.add_argument("--lr", type=float, default=2.0e-4)
    ap.add_argument("--modes", type=int, default=16)
    ap.add_argument("--seed", type=int, default=20260722)
    ap.add_argument("--checkpoint", default=None)
    args = ap.parse_args(argv)
    device = torch.device("cuda", torch.cuda.current_device())
    torch.manual_seed(args.seed)
    x_tr, y_tr = scx_data.fno_pairs_device(args.n_train, args.seed, device)
    x_te, y_te = scx_data.fno_pairs_device(args.n_test, args.seed + 1, device)
    model = fno_model.FNO2d(modes1=args.modes, modes2=args.modes, width=32, n_layers=4, in_channels=10,
                            out_channels=1).to(device)
    summary = train(model, x_tr, y_tr, x_te, y_te, epochs=args.epochs, batch_size=args.batch_size, lr=args.lr,
                    seed=args.seed, checkpoint=args.checkpoint)
    print(json.dumps({k: v for k, v in summary.items() if k != "history"}, indent=1))


if __name__ == "__main__":
    main()
