"""Batch sharding across ranks on CPU (world size 2, gloo): the host side of the multi-GPU
path.  Each rank runs the forward on its contiguous, possibly ragged, batch shard and one
gather brings the shards to rank 0; a rank that never joins the gather makes the other
rank fail within the process-group timeout instead of hanging."""

from __future__ import annotations

import os
import socket
import sys
import traceback
from pathlib import Path

import pytest
import torch
import torch.multiprocessing as mp

REPO = Path(__file__).resolve().parents[1]


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _forward_shard(x, w1, w2, m1, m2):
    sys.path.insert(0, str(REPO))
    from oracle import oracle
    return oracle.spectral_conv2d_torch(x, w1, w2, m1, m2)


def _case(batch):
    g = torch.Generator().manual_seed(11)
    x = torch.randn(batch, 3, 12, 10, generator=g)
    w1 = 0.1 * torch.rand(3, 4, 4, 5, dtype=torch.cfloat, generator=g)
    w2 = 0.1 * torch.rand(3, 4, 4, 5, dtype=torch.cfloat, generator=g)
    return x, w1, w2


def _worker(rank, world, port, batch, mode, results):
    try:
        sys.path.insert(0, str(REPO / "birensupa-spectralconv_b200"))
        import scx_dist
        os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
        scx_dist.init("gloo", timeout_s=5 if mode == "dropout" else 60)
        x, w1, w2 = _case(batch)
        lo, hi = scx_dist.shard_range(batch, world, rank)
        if mode == "dropout" and rank == 1:
            results[rank] = "left"  # leaves between steps, before the gather
            return
        y = _forward_shard(x[lo:hi], w1, w2, 4, 5)
        try:
            if mode == "into":
                # preallocated output on rank 0; rank 0's shard is computed in place
                full = torch.full((batch, 4, 12, 10), float("nan")) if rank == 0 else None
                if rank == 0:
                    full[lo:hi] = y
                    y = full[lo:hi]
                scx_dist.gather_batch_into(y, full, batch)
            else:
                full = scx_dist.gather_batch(y, batch)
        except RuntimeError as e:
            results[rank] = f"error: {type(e).__name__}"
            return
        t = scx_dist.max_over_ranks(float(rank + 1))
        if rank == 0:
            ref = torch.cat([_forward_shard(x[a:b], w1, w2, 4, 5)
                             for a, b in (scx_dist.shard_range(batch, world, r) for r in range(world))])
            results[rank] = ("ok", bool(torch.equal(full, ref)), tuple(full.shape), t)
        else:
            results[rank] = ("ok", full is None, None, t)
        torch.distributed.destroy_process_group()
    except Exception:
        results[rank] = traceback.format_exc()


def _run(world, batch, mode, join_s=90):
    ctx = mp.get_context("spawn")
    port = _free_port()
    with ctx.Manager() as manager:
        results = manager.dict()
        procs = [ctx.Process(target=_worker, args=(r, world, port, batch, mode, results)) for r in range(world)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(join_s)
        alive = [p for p in procs if p.is_alive()]
        for p in alive:
            p.kill()
        return dict(results), len(alive)


@pytest.mark.parametrize("mode", ["normal", "into"])
@pytest.mark.parametrize("batch", [4, 5])  # even and ragged (3, 2) shards
def test_sharded_forward_gathers_to_rank0(batch, mode):
    res, hung = _run(2, batch, mode)
    assert hung == 0
    assert isinstance(res[0], tuple), res[0]
    status, equal, shape, tmax = res[0]
    assert status == "ok" and equal and shape == (batch, 4, 12, 10) and tmax == 2.0
    assert res[1] == ("ok", True, None, 2.0), res[1]


def test_rank_that_never_joins_fails_the_gather_in_time():
    res, hung = _run(2, 4, "dropout", join_s=60)
    assert hung == 0, "a rank kept waiting for its missing peer"
    assert res[1] == "left"
    assert isinstance(res[0], str) and res[0].startswith("error"), res[0]


def test_chunk_ranges_cover_the_shard_in_order():
    import scx_dist

    for n in range(0, 12):
        for k in range(1, 10):
            r = scx_dist.chunk_ranges(n, k)
            assert len(r) == (min(k, n) if n else 0)
            assert [i for lo, hi in r for i in range(lo, hi)] == list(range(n))
            if r:
                sizes = [hi - lo for lo, hi in r]
                assert max(sizes) - min(sizes) <= 1 and min(sizes) >= 1
