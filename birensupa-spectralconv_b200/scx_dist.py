"""Batch sharding across ranks (one process per GPU) and the final output gather.

The SpectralConv2d / FNO forward is independent per batch item and the weights are
replicated, so the only exchange is one gather of the output shards to rank 0 (one group of
NCCL point-to-point transfers over NVLink on GPUs, gloo on CPU in the tests).  Shards are contiguous and ragged when the
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


def gather_batch_into(local: torch.Tensor, out: torch.Tensor | None, batch: int, dst: int = 0) -> None:
    """Gathers the ragged per-rank batch shards of ``local`` ([b_r, ...]) into ``out``
    ([batch, ...], preallocated on rank ``dst``; ignored elsewhere).  Only rank ``dst``
    receives: every other rank sends its shard once, straight into its contiguous slice of
    ``out``, and all transfers go in one batched group of point-to-point operations (one
    NCCL group over NVLink on GPUs).  Nothing is padded, allocated or concatenated, so the
    call can sit inside a timed step.  Rank ``dst`` may compute its own shard straight into
    its slice of ``out`` (``local`` a view of it), which saves the local copy.  Every rank
    calls it once per gather."""
    world = dist.get_world_size()
    rank = dist.get_rank()
    sizes = shard_sizes(batch, world)
    if local.shape[0] != sizes[rank]:
        raise ValueError(f"rank {rank}: shard has {local.shape[0]} items, expected {sizes[rank]}")
    if not local.is_contiguous():
        raise ValueError("the local shard must be contiguous")
    if rank == dst:
        if out is None or out.shape[0] != batch or tuple(out.shape[1:]) != tuple(local.shape[1:]):
            raise ValueError(f"rank {dst} needs an output of shape {(batch,) + tuple(local.shape[1:])}")
        if not out.is_contiguous() or out.dtype != local.dtype or out.device != local.device:
            raise ValueError("the output must be contiguous, with the shard's dtype and device")
        lo, hi = shard_range(batch, world, rank)
        if hi > lo and local.data_ptr() != out[lo:hi].data_ptr():
            out[lo:hi].copy_(local)
        ops = [dist.P2POp(dist.irecv, out[slice(*shard_range(batch, world, r))], r)
               for r in range(world) if r != dst and sizes[r] > 0]
    else:
        ops = [dist.P2POp(dist.isend, local, dst)] if sizes[rank] > 0 else []
    if ops:
        for work in dist.batch_isend_irecv(ops):
            work.wait()


def gather_batch(local: torch.Tensor, batch: int, dst: int = 0) -> torch.Tensor | None:
    """Gathers the ragged per-rank batch shards of ``local`` ([b_r, ...]) into one new
    [batch, ...] tensor on rank ``dst`` (None elsewhere), through ``gather_batch_into``."""
    out = None
    if dist.get_rank() == dst:
        out = torch.empty((batch,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    gather_batch_into(local.contiguous(), out, batch, dst)
    return out


def max_over_ranks(value: float, device: torch.device | None = None) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())
