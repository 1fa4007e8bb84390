"""Batch sharding across ranks (one process per GPU) and the final output gather.

The SpectralConv2d / FNO forward is independent per batch item and the weights are
replicated, so the only exchange is one gather of the output shards to rank 0: one group of
NCCL point-to-point transfers (``gather_batch_into``; gloo on CPU in the tests), or, on GPUs,
one peer copy per rank straight into rank 0's output over NVLink (``PeerGather``).  Shards are
contiguous and ragged when the batch does not divide: B=20 over 8 ranks -> 3,3,3,3,2,2,2,2.
"""

from __future__ import annotations

import ctypes
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


class PeerGather:
    """Gather of the ragged per-rank shards of ``local`` into ``out`` on rank ``dst`` by peer
    copies (GPUs, one process per GPU).  Built once, collectively: rank ``dst`` exports its
    preallocated ``out`` ([batch, ...]) through CUDA IPC (scx_ipc_export), every other rank
    imports it and keeps the address of its own slice.  ``push(stream)`` then copies this rank's
    shard into that slice with one device-to-device copy (copy engines, over NVLink), ordered on
    ``stream`` after the kernels that wrote ``local``; rank ``dst`` copies its shard locally
    unless ``local`` is already a view of its slice.  No collective runs per step: a push is
    complete when its stream reaches it, so the step time is the max over ranks of their
    stream times, and rank ``dst`` may read ``out`` once every rank has synchronised its
    stream and passed a host barrier (``sync()`` does both).  ``close()`` releases the import."""

    def __init__(self, local: torch.Tensor, out: torch.Tensor | None, batch: int, dst: int = 0):
        import _scx

        self.lib = _scx.lib
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        self.dst = dst
        sizes = shard_sizes(batch, self.world)
        if local.shape[0] != sizes[self.rank] or not local.is_contiguous() or local.device.type != "cuda":
            raise ValueError(f"rank {self.rank}: needs a contiguous CUDA shard of {sizes[self.rank]} items")
        self.local = local
        self.nbytes = local.numel() * local.element_size()
        item = self.nbytes // max(1, sizes[self.rank]) if sizes[self.rank] else 0
        nh = self.lib.scx_ipc_handle_bytes()
        payload = [None]
        if self.rank == dst:
            if out is None or out.shape[0] != batch or tuple(out.shape[1:]) != tuple(local.shape[1:]) \
                    or not out.is_contiguous() or out.dtype != local.dtype or out.device != local.device:
                raise ValueError(f"rank {dst} needs a contiguous output of shape {(batch,) + tuple(local.shape[1:])}")
            handle = (ctypes.c_char * nh)()
            offset = ctypes.c_ulonglong(0)
            _scx.check(self.lib.scx_ipc_export(out.data_ptr(), handle, ctypes.byref(offset)), "scx_ipc_export")
            payload = [(bytes(handle), int(offset.value), out.numel() * out.element_size() // batch)]
        dist.broadcast_object_list(payload, src=dst)
        handle_bytes, offset, item_bytes = payload[0]
        self.base = None
        lo, _ = shard_range(batch, self.world, self.rank)
        if self.rank == dst:
            self.dst_ptr = out.data_ptr() + lo * item_bytes
        else:
            base = ctypes.c_void_p(0)
            buf = (ctypes.c_char * nh).from_buffer_copy(handle_bytes)
            _scx.check(self.lib.scx_ipc_import(buf, ctypes.byref(base)), "scx_ipc_import")
            self.base = base.value
            self.dst_ptr = self.base + offset + lo * item_bytes
        if item and item != item_bytes:
            raise ValueError("shard items and output items differ in size")

    def push(self, stream: int) -> None:
        if self.nbytes and self.dst_ptr != self.local.data_ptr():
            import _scx

            _scx.check(self.lib.scx_copy_async(self.dst_ptr, self.local.data_ptr(), self.nbytes, stream),
                       "scx_copy_async")

    def push_items(self, stream: int, lo: int, hi: int) -> None:
        """Copies items [lo, hi) of this rank's shard into their slots of the output (one copy on
        ``stream``, ordered after what ``stream`` has already been given)."""
        if hi <= lo or self.nbytes == 0 or self.dst_ptr == self.local.data_ptr():
            return
        import _scx

        item = self.nbytes // self.local.shape[0]
        _scx.check(self.lib.scx_copy_async(self.dst_ptr + lo * item, self.local.data_ptr() + lo * item,
                                           (hi - lo) * item, stream), "scx_copy_async")

    def sync(self) -> None:
        torch.cuda.synchronize(self.local.device)
        dist.barrier()

    def close(self) -> None:
        if self.base is not None:
            self.lib.scx_ipc_close(self.base)
            self.base = None


def chunk_ranges(n: int, chunks: int) -> list[tuple[int, int]]:
    """[lo, hi) ranges of ``n`` items in ``min(chunks, n)`` contiguous pieces whose sizes differ
    by at most one."""
    k = max(1, min(int(chunks), int(n)))
    return [(n * i // k, n * (i + 1) // k) for i in range(k)] if n > 0 else []


# Items per sub-batch of PipelinedGather: at 256 x 256, C64, a one-item forward is latency-bound
# (eight of them took longer than the eight-item forward and its push together), two items
# keep the forward efficient while the pushes overlap.
DEFAULT_CHUNK_ITEMS = 2


class PipelinedGather:
    """SpectralConv2d forward of this rank's batch shard, then the gather of all shards to rank
    ``dst``, with the transfer overlapped with the forward.  On a rank other than ``dst`` the
    shard runs as ``chunks`` sub-batches (of ``DEFAULT_CHUNK_ITEMS`` items by default) on the
    caller's stream, and
    each sub-batch's output is pushed into its slots of ``dst``'s output by a copy on a second
    stream as soon as its forward has finished: the NVLink transfer of sub-batch k runs while
    sub-batch k + 1 is computed.  Rank ``dst`` runs its shard in one forward straight into its
    slice of ``out`` (``y`` must be that slice).  ``run(stream)`` enqueues one step and makes
    ``stream`` wait for the last push, so a step is complete when ``stream`` reaches its end; it
    can be captured in a CUDA graph once the shape has run outside a capture (the first use
    builds the twiddle tables).

    x [nb, Cin, H, W] and y [nb, Cout, H, W]: this rank's contiguous shard on its GPU; w1, w2:
    [Cin, Cout, m1, m2, 2] interleaved float32 on the same GPU; out: the preallocated
    [batch, Cout, H, W] output on rank ``dst`` (None elsewhere).  Built collectively (it builds a
    ``PeerGather``); ``close()`` releases the peer mapping."""

    def __init__(self, x: torch.Tensor, y: torch.Tensor, w1: torch.Tensor, w2: torch.Tensor, m1: int, m2: int,
                 out: torch.Tensor | None, batch: int, chunks: int | None = None, dst: int = 0):
        import _scx

        if not (x.is_cuda and y.is_cuda and x.is_contiguous() and y.is_contiguous() and x.dim() == 4 and y.dim() == 4):
            raise ValueError("x and y must be contiguous 4-D CUDA tensors")
        self.lib = _scx.lib
        self.x, self.y, self.w1, self.w2 = x, y, w1, w2
        self.nb, self.cin, self.h, self.w = (int(v) for v in x.shape)
        self.cout = int(y.shape[1])
        self.m1, self.m2 = int(m1), int(m2)
        self.peer = PeerGather(y, out, batch, dst)
        remote = self.peer.dst_ptr != y.data_ptr()
        default = max(1, -(-self.nb // DEFAULT_CHUNK_ITEMS))
        self.ranges = chunk_ranges(self.nb, (chunks or default) if remote else 1)
        self.remote = remote
        biggest = max((hi - lo for lo, hi in self.ranges), default=0)
        self.ws_bytes = self.lib.scx_spectral_conv2d_workspace_size(max(1, biggest), self.cin, self.cout, self.h,
                                                                    self.w, self.m1, self.m2)
        if self.ws_bytes == 0:
            raise ValueError("invalid SpectralConv2d sizes")
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=x.device)
        self.copy_stream = torch.cuda.Stream(x.device)
        self.x_item = x[0].numel() * x.element_size() if self.nb else 0
        self.y_item = y[0].numel() * y.element_size() if self.nb else 0

    def run(self, stream: torch.cuda.Stream) -> None:
        import _scx

        h = stream.cuda_stream
        for lo, hi in self.ranges:
            _scx.check(self.lib.scx_spectral_conv2d_fwd(self.x.data_ptr() + lo * self.x_item, self.w1.data_ptr(),
                                                        self.w2.data_ptr(), self.y.data_ptr() + lo * self.y_item,
                                                        hi - lo, self.cin, self.cout, self.h, self.w, self.m1,
                                                        self.m2, self.ws.data_ptr(), self.ws_bytes, h),
                       "scx_spectral_conv2d_fwd")
            if self.remote:
                done = torch.cuda.Event()
                done.record(stream)
                self.copy_stream.wait_event(done)
                self.peer.push_items(self.copy_stream.cuda_stream, lo, hi)
        if self.remote:
            stream.wait_stream(self.copy_stream)

    def close(self) -> None:
        self.peer.close()


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
