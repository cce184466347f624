"""Multi-GPU partitioning: one process per GPU, ``torch.distributed`` for the
plumbing (NCCL over NVLink on the B200 box, gloo in CPU tests).

The reference is single-GPU (no ``device!``, test/test_ka_upstream.jl:6-10);
this module is the partitioning layer the north star asks for in the launch
path:

* vadd, gather, histogram and mapreduce shard their index space into
  contiguous ranges ``[r*n/W, (r+1)*n/W)`` (``shard_range``); vadd and gather
  need no exchange;
* mapreduce combines one fp64 partial per rank and histogram one u32 count
  vector per rank: inside the kernel over NVLink peer memory (``PeerReduce``,
  the product path), or with a single NCCL all-reduce (``combine_partial`` /
  ``combine_counts``, kept for callers without the peer mailbox);
* the matmul shards row blocks of A (``row_block``); B is replicated.

Each function takes the process group explicitly (``None`` = the default
group) and leaves the local computation to the caller, so the same code runs
with NCCL device tensors and gloo host tensors.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

_REDUCE_OPS = {"add": dist.ReduceOp.SUM, "mul": dist.ReduceOp.PRODUCT,
               "max": dist.ReduceOp.MAX, "min": dist.ReduceOp.MIN}


def world(group=None) -> tuple[int, int]:
    """(rank, world_size) of this process, (0, 1) without a process group."""
    if not dist.is_available() or not dist.is_initialized():
        return 0, 1
    return dist.get_rank(group), dist.get_world_size(group)


def shard_range(n: int, rank: int, world_size: int) -> tuple[int, int]:
    """Contiguous shard ``[lo, hi)`` of ``n`` elements for ``rank``; the first
    ``n % world_size`` ranks hold one extra element."""
    if world_size < 1 or not 0 <= rank < world_size:
        raise ValueError(f"bad rank {rank} for world size {world_size}")
    base, extra = divmod(n, world_size)
    lo = rank * base + min(rank, extra)
    return lo, lo + base + (1 if rank < extra else 0)


def row_block(m: int, rank: int, world_size: int, align: int = 128) -> tuple[int, int]:
    """Row range of A (and C) owned by ``rank`` for the sharded matmul, in
    multiples of ``align`` rows except for the last rank."""
    blocks = -(-m // align)
    lo_b, hi_b = shard_range(blocks, rank, world_size)
    return min(lo_b * align, m), min(hi_b * align, m)


def combine_partial(partial: torch.Tensor, op: str = "add", group=None) -> torch.Tensor:
    """All-reduce a per-rank reduction partial in place (one fp64 scalar for
    ``sum(x.^2)``): the single exchange step of the sharded mapreduce."""
    if world(group)[1] > 1:
        dist.all_reduce(partial, op=_REDUCE_OPS[op], group=group)
    return partial


def combine_counts(counts: torch.Tensor, group=None) -> torch.Tensor:
    """All-reduce per-rank histogram counts in place.  u32 counts travel as
    int32: two's-complement addition is addition mod 2^32, so the bits equal a
    u32 sum with wrap-around."""
    if counts.dtype not in (torch.int32, torch.int64):
        raise TypeError(f"counts must be int32 storage, got {counts.dtype}")
    if world(group)[1] > 1:
        dist.all_reduce(counts, op=dist.ReduceOp.SUM, group=group)
    return counts


def barrier(group=None, device: torch.device | None = None) -> None:
    if world(group)[1] > 1:
        if device is not None and device.type == "cuda":
            dist.barrier(group=group, device_ids=[device.index])
        else:
            dist.barrier(group=group)


def exchange_bytes(mine: bytes, group=None) -> list[bytes]:
    """All-gather one small byte string per rank (rank order)."""
    rank, size = world(group)
    if size == 1:
        return [mine]
    out: list = [None] * size
    dist.all_gather_object(out, mine, group=group)
    return list(out)


class PeerReduce:
    """Fused multi-GPU mapreduce: one launch per rank computes the local
    reduction and exchanges the fp64 partial with every other rank through
    CUDA-IPC-mapped peer memory (``mk_mapreduce_f32_allreduce``); no NCCL call
    per reduction.  Create it collectively (every rank of ``group``, each on
    its own GPU); every rank must then call ``__call__`` equally often."""

    def __init__(self, group=None):
        import ctypes as C

        from . import _lib
        self._lib = _lib
        rank, size = world(group)
        if size < 2:
            raise ValueError("PeerReduce needs a process group of at least 2 ranks")
        L = _lib.lib()
        hs = L.mk_peer_handle_size()
        buf = C.create_string_buffer(hs)
        _lib.check(L.mk_peer_create(size, rank, buf), "mk_peer_create")
        handles = exchange_bytes(buf.raw, group)
        allh = C.create_string_buffer(b"".join(handles), hs * size)
        _lib.check(L.mk_peer_connect(allh), "mk_peer_connect")
        self.rank, self.size = rank, size

    def __call__(self, x, f: str = "abs2", op: str = "add", init: float = 0.0,
                 out: torch.Tensor | None = None) -> torch.Tensor:
        """Global ``mapreduce(f, op, x)`` over all ranks' shards, as a
        1-element fp64 device tensor on every rank (asynchronous)."""
        from .array import current_stream_handle
        L = self._lib.lib()
        if out is None:
            out = torch.empty(1, dtype=torch.float64, device=x.storage.device)
        self._lib.check(L.mk_mapreduce_f32_allreduce(out.data_ptr(), x.pointer(), x.length,
                                                     self._lib.MK_F[f], self._lib.MK_OP[op], float(init),
                                                     current_stream_handle()), "mapreduce allreduce")
        return out

    def submit(self, x, out: torch.Tensor, f: str = "abs2", op: str = "add", init: float = 0.0) -> torch.Tensor:
        """Pipelined ``__call__`` (``mk_mapreduce_f32_allreduce_async``): the
        global result lands in ``out`` once the next ``submit``/``__call__``
        or ``complete()`` has run on the stream; no rank waits for its peers
        inside the step.  ``out`` must stay alive until then."""
        from .array import current_stream_handle
        L = self._lib.lib()
        self._lib.check(L.mk_mapreduce_f32_allreduce_async(out.data_ptr(), x.pointer(), x.length,
                                                           self._lib.MK_F[f], self._lib.MK_OP[op], float(init),
                                                           current_stream_handle()), "mapreduce allreduce async")
        return out

    def complete(self) -> None:
        """Write the last pending ``submit`` result (asynchronous)."""
        from .array import current_stream_handle
        self._lib.check(self._lib.lib().mk_allreduce_complete(current_stream_handle()), "allreduce complete")

    def histogram(self, counts, keys, out: torch.Tensor, nbins: int | None = None, pipelined: bool = False):
        """Fused multi-GPU histogram (``mk_hist_u32_allreduce[_async]``):
        accumulate this rank's 1-based Int32 ``keys`` into its UInt32
        ``counts`` and write the sum of every rank's counts into ``out`` (a
        separate int32/uint32 device tensor of ``nbins`` elements), all in one
        launch.  ``pipelined=True`` defers ``out`` to the next exchanging
        histogram call or ``hist_complete()``."""
        from .array import current_stream_handle
        L = self._lib.lib()
        nb = counts.length if nbins is None else nbins
        fn = L.mk_hist_u32_allreduce_async if pipelined else L.mk_hist_u32_allreduce
        self._lib.check(fn(out.data_ptr(), counts.pointer(), nb, keys.pointer(), keys.length,
                           current_stream_handle()), "histogram allreduce")
        return out

    def hist_complete(self) -> None:
        """Write the last pending pipelined histogram result (asynchronous)."""
        from .array import current_stream_handle
        self._lib.check(self._lib.lib().mk_hist_allreduce_complete(current_stream_handle()), "hist complete")

    def close(self) -> None:
        self._lib.check(self._lib.lib().mk_peer_destroy(), "mk_peer_destroy")


_shared_peer: PeerReduce | None = None


def shared_peer(group=None) -> PeerReduce:
    """The process's one peer mailbox (a device holds one at a time): created
    collectively on first use, then reused by every fused multi-GPU call."""
    global _shared_peer
    if _shared_peer is None:
        _shared_peer = PeerReduce(group)
    return _shared_peer
