"""Batch sharding across ranks (one process per GPU) and the final output gather.

The SpectralConv2d / FNO forward is independent per batch item and the weights are
replicated, so the only exchange is one gather of the output shards (NCCL over
NVLink on GPUs, gloo on CPU in the tests).  Shards are contiguous and ragged when the
batch does not divide: B=20 over 8 ranks -> 3,3,3,3,2,2,2,2.
"""

from __future__ import annotations

import datetime
import os

import torch
import torch.distributed as dist


def shard_sizes(batch: int, world: int) -> list[int]:
    base, extra = divmod(int(batch), int(world))
    return [base + (1 if r < extra else 0) for r in range(world)]


def shard_range(batch: int, world: int, rank: int) -> tuple[int, int]:
    sizes = shard_sizes(batch, world)
    start = sum(sizes[:rank])
    return start, start + sizes[rank]


def env_rank() -> tuple[int, int, int]:
    """(rank, local_rank, world_size) from the torchrun environment (1 process if unset)."""
    return (int(os.environ.get("RANK", 0)), int(os.environ.get("LOCAL_RANK", 0)),
            int(os.environ.get("WORLD_SIZE", 1)))


def init(backend: str, timeout_s: float = 120.0, device: torch.device | None = None) -> None:
    """Process group over 127.0.0.1 defaults with a bounded timeout, so that ranks
    waiting on a missing peer end with an error instead of hanging.  ``device`` binds an
    NCCL group to this rank's GPU."""
    os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
    os.environ.setdefault("MASTER_PORT", "29531")
    if not dist.is_initialized():
        kwargs = {"device_id": device} if device is not None and device.type == "cuda" else {}
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)


def gather_batch(local: torch.Tensor, batch: int, dst: int = 0) -> torch.Tensor | None:
    """Gathers the ragged per-rank batch shards of ``local`` ([b_r, ...]) into one
    [batch, ...] tensor on rank ``dst`` (None elsewhere).  Every rank pads its shard to
    the largest shard and joins one all_gather_into_tensor; all ranks take the same
    collective steps in the same order."""
    world = dist.get_world_size()
    rank = dist.get_rank()
    sizes = shard_sizes(batch, world)
    if local.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank}: shard has {local.shape[0]} items, expected {sizes[rank]}")
    bmax = max(sizes)
    tail = tuple(local.shape[1:])
    if local.shape[0] == bmax:
        padded = local.contiguous()
    else:
        padded = torch.zeros((bmax,) + tail, dtype=local.dtype, device=local.device)
        padded[: local.shape[0]] = local
    stacked = torch.empty((world * bmax,) + tail, dtype=local.dtype, device=local.device)
    dist.all_gather_into_tensor(stacked, padded)
    if rank != dst:
        return None
    parts = [stacked[r * bmax: r * bmax + sizes[r]] for r in range(world)]
    return torch.cat(parts, dim=0)


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
