"""The N>1 host path on CPU: world_size-2 gloo process groups exercise the
sharding + single all-reduce combine of the multi-GPU layer.  The local
per-shard computation is done by the CPU oracle here (the GPU kernels are the
-m gpu tests); what is under test is the partitioning and the exchange."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle
from cutilecpu_b200 import distributed


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        r = np.random.Generator(np.random.Philox(11))
        n = 10_007
        x = (r.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
        lo, hi = distributed.shard_range(n, rank, world)
        part = torch.tensor([oracle.sum_sq(x[lo:hi])], dtype=torch.float64)
        distributed.combine_partial(part, "add")
        mx = torch.tensor([oracle.mapreduce(x[lo:hi], "identity", "max", -np.inf)], dtype=torch.float64)
        distributed.combine_partial(mx, "max")

        keys = r.integers(1, 65, size=n, dtype=np.int32)
        counts, rc = oracle.hist(keys[lo:hi], 64)
        assert rc == 0
        ct = torch.from_numpy(counts.view(np.int32).copy())
        distributed.combine_counts(ct)

        # u32 wrap-around survives the int32 transport
        wrap = torch.from_numpy(np.array([0xFFFFFFFF, 1], dtype=np.uint32).view(np.int32).copy())
        distributed.combine_counts(wrap)
        distributed.barrier()
        if rank == 0:
            results["sum_sq"] = part.item()
            results["max"] = mx.item()
            results["counts"] = ct.numpy().view(np.uint32).copy()
            results["wrap"] = wrap.numpy().view(np.uint32).copy()
            results["ref_sum_sq"] = oracle.sum_sq(x)
            results["ref_max"] = float(x.max())
            results["ref_counts"] = np.bincount(keys - 1, minlength=64).astype(np.uint32)
    finally:
        dist.destroy_process_group()


def test_gloo_world2_combine():
    mgr = mp.Manager()
    results = mgr.dict()
    port = _free_port()
    mp.spawn(_worker, args=(2, port, results), nprocs=2, join=True)
    assert results["sum_sq"] == pytest.approx(results["ref_sum_sq"], rel=1e-12)
    assert results["max"] == results["ref_max"]
    np.testing.assert_array_equal(results["counts"], results["ref_counts"])
    np.testing.assert_array_equal(results["wrap"], np.array([0xFFFFFFFE, 2], dtype=np.uint32))


def _exchange_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        got = distributed.exchange_bytes(bytes([rank]) * 64)
        results[rank] = [bytes(g) for g in got]
    finally:
        dist.destroy_process_group()


def test_gloo_handle_exchange_rank_order():
    """The IPC-handle exchange of the fused multi-GPU reduction returns every
    rank's bytes in rank order on every rank."""
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_exchange_worker, args=(2, _free_port(), results), nprocs=2, join=True)
    for r in range(2):
        assert results[r] == [bytes([0]) * 64, bytes([1]) * 64]
