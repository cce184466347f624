"""Fused multi-GPU mapreduce over CUDA-IPC peer mailboxes
(mk_mapreduce_f32_allreduce): two processes, one GPU each.  Needs >= 2 GPUs;
with fewer it is skipped (the host logic is covered by the gloo tests)."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cutilecpu_b200 as mk
    import oracle
    from cutilecpu_b200 import distributed
    try:
        shards = [(np.random.Generator(np.random.Philox(100 + r)).random((1 << 22) + 17 * r, dtype=np.float32)
                   * 2 - 1).astype(np.float32) for r in range(world)]
        x = mk.MLIRArray(shards[rank])
        pr = distributed.PeerReduce()
        vals = []
        for it in range(6):  # several epochs, alternating ops and parity slots
            op = "add" if it % 2 == 0 else "max"
            f = "abs2" if op == "add" else "identity"
            init = 0.0 if op == "add" else -np.inf
            vals.append(pr(x, f, op, init).item())
        # pipelined form: 9 calls in flight, completed at the end, mixed with
        # a blocking call in the middle (which completes the pending one)
        outs = [torch.full((1,), float("nan"), dtype=torch.float64, device="cuda") for _ in range(9)]
        for it, o in enumerate(outs):
            op = "add" if it % 3 else "max"
            f = "abs2" if op == "add" else "identity"
            init = 0.0 if op == "add" else -np.inf
            if it == 4:
                pr(x, f, op, init, out=o)
            else:
                pr.submit(x, o, f, op, init)
        pr.complete()
        pr.complete()  # nothing pending: a no-op
        piped = [o.item() for o in outs]
        # the exchange keeps its epochs and pending result in device memory, so
        # pipelined calls captured in a CUDA graph can be replayed
        gouts = [torch.full((1,), float("nan"), dtype=torch.float64, device="cuda") for _ in range(3)]
        cap = torch.cuda.Stream()  # warmed first: per-stream scratch is allocated on first use, not in capture
        with torch.cuda.stream(cap):
            pr.submit(x, gouts[0])
            pr.complete()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for o in gouts:
                pr.submit(x, o)
            pr.complete()
        graphed = []
        for _ in range(3):
            for o in gouts:
                o.fill_(float("nan"))
            g.replay()
            graphed.append([o.item() for o in gouts])
        poll = mk._lib.lib().mk_error_poll(torch.cuda.current_stream().cuda_stream)
        pr.close()
        full = np.concatenate(shards)
        results[rank] = {"vals": vals, "piped": piped, "graphed": graphed, "poll": poll, "sum": oracle.sum_sq(full),
                         "max": float(full.max())}
    finally:
        dist.destroy_process_group()


def _hist_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cutilecpu_b200 as mk
    import oracle
    from cutilecpu_b200 import distributed, workloads
    try:
        be = mk.MLIRCUDABackend()
        nb = 4096
        keys_h = [workloads.zipf_keys((1 << 22) + 5 * r, nb, 1.1, stream=30 + 100 * r) for r in range(world)]
        keys = mk.MLIRArray(keys_h[rank])
        pr = distributed.PeerReduce()
        got = []
        # blocking, then 5 pipelined steps (counts re-zeroed each step), a
        # blocking step in the middle completing the pending one, then complete
        outs = [torch.full((nb,), -1, dtype=torch.int32, device="cuda") for _ in range(7)]
        for it, o in enumerate(outs):
            counts = mk.zeros(be, "UInt32", nb)
            pr.histogram(counts, keys, o, pipelined=it not in (0, 3))
        pr.hist_complete()
        pr.hist_complete()  # nothing pending: a no-op
        got = [o.cpu().numpy().view(np.uint32) for o in outs]
        # captured in a CUDA graph (counts zeroed inside), replayed twice
        counts = mk.zeros(be, "UInt32", nb)
        gouts = [torch.full((nb,), -1, dtype=torch.int32, device="cuda") for _ in range(2)]
        cap = torch.cuda.Stream()
        with torch.cuda.stream(cap):
            counts.storage.zero_()
            pr.histogram(counts, keys, gouts[0], pipelined=True)
            pr.hist_complete()
        torch.cuda.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=cap):
            for o in gouts:
                counts.storage.zero_()
                pr.histogram(counts, keys, o, pipelined=True)
            pr.hist_complete()
        for _ in range(2):
            for o in gouts:
                o.fill_(-1)
            g.replay()
            got += [o.cpu().numpy().view(np.uint32) for o in gouts]
        poll = mk._lib.lib().mk_error_poll(torch.cuda.current_stream().cuda_stream)
        pr.close()
        want = sum(oracle.hist(k, nb)[0].astype(np.int64) for k in keys_h).astype(np.uint32)
        results[rank] = {"ok": all(np.array_equal(g, want) for g in got), "poll": poll}
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_histogram_two_gpus(cuda):
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_hist_worker, args=(2, _port(), results), nprocs=2, join=True)
    for r in (0, 1):
        assert results[r]["poll"] == 0
        assert results[r]["ok"]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allreduce_two_gpus(cuda):
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_worker, args=(2, _port(), results), nprocs=2, join=True)
    r0, r1 = results[0], results[1]
    assert r0["poll"] == 0 and r1["poll"] == 0
    assert r0["vals"] == r1["vals"]  # bit-identical on every rank
    for it, v in enumerate(r0["vals"]):
        if it % 2 == 0:
            assert v == pytest.approx(r0["sum"], rel=1e-5)
        else:
            assert v == r0["max"]
    assert r0["piped"] == r1["piped"]
    assert r0["graphed"] == r1["graphed"]
    for rep in r0["graphed"]:
        assert rep == [r0["vals"][0]] * 3  # every replay, bit-identical to the eager blocking form
    for it, v in enumerate(r0["piped"]):
        if it % 3:
            assert v == r0["vals"][0]  # bit-identical to the blocking form
        else:
            assert v == r0["max"]


def _timeout_worker(rank, world, port, results):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["MK_WAIT_LIMIT_CYCLES"] = str(200_000_000)  # ~0.1 s: a short, bounded wait
    torch.cuda.set_device(rank)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    import cutilecpu_b200 as mk
    from cutilecpu_b200 import distributed
    try:
        x = mk.MLIRArray(np.ones(1 << 20, dtype=np.float32))
        pr = distributed.PeerReduce()
        rc = 0
        if rank == 0:  # rank 1 never joins this reduction: rank 0's wait must run out
            v = pr(x).item()
            rc = mk._lib.lib().mk_error_poll(torch.cuda.current_stream().cuda_stream)
            results["v"] = v
        dist.barrier()  # rank 1 keeps its mailbox mapped until rank 0 is done
        pr.close()
        results[rank] = rc
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_fused_allreduce_missing_rank_times_out(cuda):
    """Failure detection without a GPU fault: a rank that does not arrive makes
    the bounded in-kernel wait give up; the status is MK_ERR_TIMEOUT and the
    GPU stays usable."""
    mgr = mp.Manager()
    results = mgr.dict()
    mp.spawn(_timeout_worker, args=(2, _port(), results), nprocs=2, join=True)
    from cutilecpu_b200 import _lib
    assert results[0] == _lib.MK_ERR_TIMEOUT
    assert results[1] == 0
