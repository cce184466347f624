#!/usr/bin/env python
"""Benchmark of the MLIRKernels.jl hot path on B200: HBM GB/s of the fused
mapreduce ``sum(x.^2)`` over 2^28 Float32 (the BASELINE configuration the
metric is quoted on), plus the other four kernels with ``--kernel``.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--kernel reduce|vadd|gather|histogram|matmul_simt|all]

One process per GPU (torchrun for N > 1, NCCL).  Per-GPU work is fixed
(weak scaling): every rank holds its own contiguous shard of the size the
configuration names.  A step is one pass of the kernel over its shard, plus the
single NCCL all-reduce of the partial where the path has one (reduce,
histogram).  Rank 0 prints one JSON line per kernel.

``--impl reference`` times the reference's CPU execution model (the restated
MLIRBackend of oracle/oracle.c, all host threads) on the same configuration;
rank 0 alone runs it.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import operator
import os
import shutil
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

HBM_FALLBACK_GBS = 6650.0
L2_BYTES = 126 * 2**20


def peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except Exception:
            pass
    return HBM_FALLBACK_GBS, "fallback"


def tensor_peak() -> tuple[float, str]:
    """3xTF32 roofline: dense TF32 runs at half the bf16 rate and every fp32
    product costs three TF32 products, so peak = bf16 / 2 / 3."""
    p = ROOT / "MEASURED_PEAKS.json"
    bf16, kind = 1590.0, "fallback"
    if p.exists():
        try:
            bf16, kind = float(json.loads(p.read_text())["bf16_tflops"]), "measured"
        except Exception:
            pass
    return round(bf16 / 6.0, 2), f"{kind} bf16 burst / 2 (tf32) / 3 (3xTF32)"


# ----------------------------------------------------------------- clocks --

class ClockSampler:
    """nvidia-smi samples of SM clock and throttle reasons during a region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, device_index: int):
        self.dev = device_index
        self.proc = None
        self.path = None

    def start(self):
        exe = shutil.which("nvidia-smi")
        if exe is None:
            return self
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        self.fh = open(self.path, "w")
        self.proc = subprocess.Popen([exe, f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                      "-i", str(self.dev), "-lms", "50"], stdout=self.fh,
                                     stderr=subprocess.DEVNULL)
        # nvidia-smi needs up to a second before its first sample: wait for it
        # so that a short region (the GEMM's 20 steps take ~85 ms) is sampled
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            self.fh.flush()
            if Path(self.path).read_text().count("\n") >= 1:
                break
            time.sleep(0.02)
        self.skip = Path(self.path).read_text().count("\n")  # samples taken before the region
        return self

    def stop(self) -> dict | None:
        if self.proc is None:
            return None
        time.sleep(0.06)  # one more sampling period
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        self.fh.close()
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [x.strip() for x in line.split(",")]
            if len(parts) >= 9:
                rows.append(parts)
        os.unlink(self.path)
        if len(rows) > self.skip:
            rows = rows[self.skip:]
        else:
            rows = rows[-1:]  # region shorter than one period: the sample nearest its end
        if not rows:
            return None
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[5 + i].lower() == "active"})
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ configs -----

# The five BASELINE configurations in the order the default run times them;
# the mapreduce, the configuration the headline metric is quoted on, is last.
BASELINE_KINDS = ["vadd", "gather", "histogram", "matmul", "reduce"]

_WORKLOAD_TEXT = {
    "reduce": ("mapreduce sum(x.^2), Float32 x ~ U[-1,1), n=2^28 per GPU (configs[1]), rel 1e-5 of fp64; "
               "N>1: one global sum over all ranks' shards per step",
               "input (1 GiB) larger than L2; no flush"),
    "maximum": ("maximum(x) via mapreducedim!, Float32 x ~ U[-1,1), n=2^28 per GPU (scope row f1); Julia max "
                "semantics, exact", "input (1 GiB) larger than L2; no flush"),
    "findmax": ("findmax(x) (value, first 1-based index), Float32 x ~ U[-1,1), n=2^28 per GPU (scope row f1); "
                "Julia order: NaN wins, +0 above -0, first index", "input (1 GiB) larger than L2; no flush"),
    "vadd": ("vadd c=a+b Float32 n=2^20 per GPU (configs[0])",
             "24 rotating a/b/c sets (302 MB, larger than L2): every step reads inputs from HBM; no flush"),
    "gather": ("gather c=a[idx] Float32 a 2^27 (replicated on every GPU), Int32 idx 2^27 per GPU uniform in "
               "[1,2^27] (configs[2])", "inputs (1.5 GiB) larger than L2; no flush"),
    "gather_ceiling": ("random 4-byte reads of a 2^27 Float32 array at hashed positions, 2^27 per GPU, no index "
                       "stream, one u32 checksum per block (device random-read ceiling for configs[2])",
                       "array (512 MiB) larger than L2; no flush"),
    "histogram": ("histogram Int32 keys 2^26 per GPU ~ Zipf(1.1) on 1..4096, UInt32 counts (configs[3]); counts "
                  "zeroed each step; N>1: global counts over all ranks' keys per step",
                  "input (256 MiB) larger than L2; no flush"),
    "matmul": ("mm_tiled! C=A*B Float32 8192^3 per GPU (configs[4]), fp32 result within rel 1e-5 of fp64; "
               "N>1: rank r owns row block r of an (8192N)x8192 A, B replicated", "operands larger than L2"),
    "matmul_simt": ("mm_tiled! 16x16 SIMT, Float32 8192^3 per GPU (configs[4])", "operands larger than L2"),
    "scan": ("cumsum of Float32 x ~ U[0,1), n=2^28 per GPU (scope row f2: AK.accumulate!)",
             "input (1 GiB) larger than L2; no flush"),
    "reduce_dims": ("sum(m; dims=1) of a 16384x16384 Float32 matrix per GPU (scope row f1: dims reductions)",
                    "input (1 GiB) larger than L2; no flush"),
}


# How this library computes each workload (printed as "impl_notes" on its own
# lines only; the reference arm computes the same workload its own way).
IMPL_NOTES = {
    "reduce": "fused single pass, fp64 accumulation; N>1: each step's kernel publishes its fp64 partial to "
              "every rank over NVLink peer memory and folds the previous step's global result (pipelined, "
              "no NCCL call); the last step's result is completed inside the timed region; the K steps run "
              "as one CUDA graph",
    "matmul": "tcgen05 3xTF32 (TMEM accumulators, TMA-fed, CTA pairs); the split pre-pass is inside the step",
    "histogram": "per-block shared-memory bins, flushed with global atomics; N>1: the same launch publishes the "
                 "4096 counts (epoch-tagged words) to every rank over NVLink and folds the previous step's global "
                 "counts (pipelined, no NCCL call); the K steps (counts zeroed, histogram) run as one CUDA graph",
    "gather": "16-byte index/output streams, 8 random 4-byte loads in flight per thread",
    "vadd": "16-byte loads/stores, grid of resident blocks, programmatic dependent launch; the K timed steps "
            "run as one CUDA graph",
}


def config_of(kind: str, world: int, n_override: int | None = None) -> dict:
    """The ``config`` object of a kernel's JSON line.  Both arms print the same
    one for the same N, so a run pair compares like with like."""
    from cutilecpu_b200 import workloads
    text, l2 = _WORKLOAD_TEXT[kind]
    c: dict = {"workload": text}
    base = workloads.CONFIGS
    if kind in ("matmul", "matmul_simt"):
        m = n_override or base["matmul"]["m"]
        c.update(m=m, n=n_override or base["matmul"]["n"], k=n_override or base["matmul"]["k"])
    elif kind == "reduce_dims":
        r = n_override or (1 << 14)
        c.update(rows=r, cols=r)
    else:
        src = {"maximum": "reduce", "findmax": "reduce", "gather_ceiling": "gather", "scan": None}.get(kind, kind)
        c["n_per_gpu"] = n_override or (base[src]["n"] if src else 1 << 28)
    c["l2"] = l2
    c["parallelism"] = f"dp{world} (contiguous shards)" if world > 1 else "single GPU"
    if n_override:
        c["workload"] = "REDUCED SIZE (profiling case, not a benchmark line): " + c["workload"]
    return c


# ----------------------------------------------------------- workloads -----

class Workload:
    """One benchmark configuration on one rank."""

    name = ""
    metric = ""
    unit = "GB/s"
    dtype = "f32"

    def __init__(self, rank: int, world: int):
        self.rank, self.world = rank, world

    def prepare(self, slot=0):
        """Per-step set-up that is not the kernel (runs inside the timed step,
        outside the kernel's own events)."""

    # algorithmic units per step on this rank (bytes, or flops)
    units_per_step = 0.0
    launches_per_step = 1
    needs_l2_flush = False
    h2d_bytes = 0
    d2h_bytes = 0


def _dist_allreduce_max(x: float) -> float:
    import torch
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return t.item()
    return x


class CheckFailed(AssertionError):
    """A benchmarked configuration's result differs from the oracle."""


def dev_sms() -> int:
    import torch
    return torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count


def _dist_gather_f64(x: float) -> list[float]:
    """Every rank's value, in rank order (a one-element list at N=1)."""
    import torch
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        out = [torch.empty_like(t) for _ in range(dist.get_world_size())]
        dist.all_gather(out, t)
        return [o.item() for o in out]
    return [x]


def _dist_sum_f64(x: float) -> float:
    import torch
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.item()
    return x


def _dist_sum_i64(a: np.ndarray) -> np.ndarray:
    import torch
    import torch.distributed as dist
    if dist.is_initialized() and dist.get_world_size() > 1:
        t = torch.from_numpy(np.ascontiguousarray(a, dtype=np.int64)).cuda()
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return t.cpu().numpy()
    return a


def make_workload(kind: str, rank: int, world: int, n_override: int | None = None):
    import torch

    import cutilecpu_b200 as mk
    from cutilecpu_b200 import _lib, distributed, workloads

    L = _lib.lib()
    be = mk.MLIRCUDABackend()
    stream = lambda: torch.cuda.current_stream().cuda_stream  # noqa: E731

    class Reduce(Workload):
        name = "reduce"
        metric = "mapreduce sum(x.^2) HBM GB/s"
        cfg = workloads.CONFIGS["reduce"]
        graph_steps = True     # the K steps (and, at N>1, the completion) as one CUDA graph
        kernel_events = True   # plus an eager pass for the kernel's own duration

        def __init__(self):
            super().__init__(rank, world)
            n = self.n = n_override or self.cfg["n"]
            self.x_host = workloads.uniform_pm1(n, stream=1 + 100 * rank)
            self.x = mk.MLIRArray(self.x_host)
            self.out = torch.empty(1, dtype=torch.float64, device="cuda")
            self.peer = distributed.shared_peer() if world > 1 else None
            self.outs = [torch.empty(1, dtype=torch.float64, device="cuda") for _ in range(2)]
            self.step_no = 0
            self.units_per_step = 4.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 8

        def launch(self):
            if self.peer is not None:
                # fused and pipelined: the local reduction publishes its fp64
                # partial over NVLink and folds the previous step's global
                # result, all in one launch; no rank waits for a peer inside
                # a step
                self.step_no += 1
                _lib.check(L.mk_mapreduce_f32_allreduce_async(self.outs[self.step_no % 2].data_ptr(),
                                                              self.x.pointer(), self.n, 1, 0, 0.0, stream()),
                           "sum_sq allreduce")
            else:
                _lib.check(L.mk_sum_sq_f32(self.out.data_ptr(), self.x.pointer(), self.n, stream()), "sum_sq")

        def combine(self):
            pass  # the exchange is inside the kernel

        def extra_roofline(self, K, kern_ms):
            """N>1: where the fused exchange's time goes, from device-clock
            stamps of K pipelined steps (mk_peer_trace): the streaming part
            (kernel start to the last block's exchange), publishing the
            partial to every rank, and folding the previous step's result
            (which includes any wait for a late peer).  Medians per rank, then
            the max over ranks."""
            if self.peer is None:
                return {}
            log = torch.zeros(4 * K, dtype=torch.int64, device="cuda")
            _lib.check(L.mk_peer_trace(log.data_ptr(), K), "trace")
            for _ in range(K):
                self.launch()
            self.finish()
            torch.cuda.synchronize()
            _lib.check(L.mk_peer_trace(None, 0), "trace off")
            t = log.cpu().numpy().view(np.uint64).reshape(K, 4).astype(np.int64)
            parts = {"stream_us": t[:, 1] - t[:, 0], "publish_us": t[:, 2] - t[:, 1], "fold_us": t[:, 3] - t[:, 2]}
            return {"exchange_trace": {k: round(_dist_allreduce_max(float(np.median(v)) * 1e-3), 2)
                                       for k, v in parts.items()} | {"kernel_us": round(kern_ms * 1e3, 2)}}

        def finish(self):
            """Completes the last pending global result (timed: it is inside
            the region, after the last step)."""
            if self.peer is not None:
                _lib.check(L.mk_allreduce_complete(stream()), "allreduce complete")
                self.out = self.outs[self.step_no % 2]

        def check(self):
            # every N: the fused result against the fp64 oracle of all shards,
            # and the same bits on every rank
            import oracle
            got = self.out.item()
            want = _dist_sum_f64(oracle.sum_sq(self.x_host))
            if not abs(got - want) <= 1e-5 * abs(want):
                raise CheckFailed(f"reduce: rank {rank} got {got!r}, oracle {want!r}")
            if _dist_allreduce_max(got) != -_dist_allreduce_max(-got):
                raise CheckFailed(f"reduce: ranks disagree (rank {rank} has {got!r})")

        def e2e_setup(self):
            self.pinned = torch.from_numpy(self.x_host).pin_memory()
            self.xd = mk.allocate(be, "Float32", self.n)

        def e2e_step(self):
            mk.copyto(be, self.xd, self.pinned)
            if self.peer is not None:
                res = self.peer(self.xd, "abs2", "add")
            else:
                res = mk.reductions.mapreduce_device(mk.abs2, operator.add, self.xd)
            return res.item()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            tmp = np.empty(self.n + self.n // 512 + 2, dtype=np.float32)
            return lambda: Lo.mlirb_sum_sq_f32(self.x_host.ctypes.data, self.n, 256, tmp.ctypes.data), \
                self.units_per_step, "full 2^28-element sum(x.^2): materialised x.^2 + fp32 block-tree rounds"

    class Maximum(Workload):
        name = "maximum"
        metric = "maximum(x) HBM GB/s"
        cfg = workloads.CONFIGS["reduce"]

        def __init__(self):
            super().__init__(rank, world)
            n = self.n = n_override or self.cfg["n"]
            self.x_host = workloads.uniform_pm1(n, stream=3 + 100 * rank)
            self.x = mk.MLIRArray(self.x_host)
            self.out = torch.empty(1, dtype=torch.float64, device="cuda")
            self.units_per_step = 4.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 8

        def launch(self):
            _lib.check(L.mk_mapreduce_f32(self.out.data_ptr(), self.x.pointer(), self.n, 0, 1, float("-inf"),
                                          stream()), "maximum")

        def combine(self):
            pass

        def check(self):
            assert self.out.item() == float(self.x_host.max())

        def e2e_setup(self):
            self.pinned = torch.from_numpy(self.x_host).pin_memory()
            self.xd = mk.allocate(be, "Float32", self.n)

        def e2e_step(self):
            mk.copyto(be, self.xd, self.pinned)
            return mk.maximum(self.xd)

        def cpu_sample(self, threads):
            import ctypes as C
            import oracle
            Lo = oracle.lib()
            v = C.c_double()
            return lambda: Lo.mlirb_findext_f32(C.byref(v), self.x_host.ctypes.data, self.n, 1), \
                self.units_per_step, "full 2^28-element maximum (Julia order), OpenMP chunks + ordered combine"

    class FindMax(Workload):
        name = "findmax"
        metric = "findmax(x) HBM GB/s"
        cfg = workloads.CONFIGS["reduce"]

        def __init__(self):
            super().__init__(rank, world)
            n = self.n = n_override or self.cfg["n"]
            self.x_host = workloads.uniform_pm1(n, stream=4 + 100 * rank)
            self.x = mk.MLIRArray(self.x_host)
            self.val = torch.empty(1, dtype=torch.float64, device="cuda")
            self.idx = torch.empty(1, dtype=torch.int64, device="cuda")
            self.units_per_step = 4.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 16

        def launch(self):
            _lib.check(L.mk_findext_f32(self.val.data_ptr(), self.idx.data_ptr(), self.x.pointer(), self.n, 1,
                                        stream()), "findmax")

        def combine(self):
            pass

        def check(self):
            import oracle
            assert (self.val.item(), self.idx.item()) == oracle.findext(self.x_host, True)

        def e2e_setup(self):
            self.pinned = torch.from_numpy(self.x_host).pin_memory()
            self.xd = mk.allocate(be, "Float32", self.n)

        def e2e_step(self):
            mk.copyto(be, self.xd, self.pinned)
            return mk.findmax(self.xd)

        def cpu_sample(self, threads):
            import ctypes as C
            import oracle
            Lo = oracle.lib()
            v = C.c_double()
            return lambda: Lo.mlirb_findext_f32(C.byref(v), self.x_host.ctypes.data, self.n, 1), \
                self.units_per_step, "full 2^28-element findmax, OpenMP chunks + ordered combine"

    class Vadd(Workload):
        name = "vadd"
        metric = "vadd HBM GB/s"
        cfg = workloads.CONFIGS["vadd"]
        # A 12 MiB vadd is launch-bound: the timed steps run as one CUDA graph
        # of K launches (programmatic dependent launch between them), each
        # step on the next of SETS input/output sets, which together exceed
        # L2, so every step reads a and b from HBM without a flush kernel.
        graph_steps = True
        SETS = 24

        def __init__(self):
            super().__init__(rank, world)
            n = self.n = n_override or self.cfg["n"]
            self.a_host = workloads.uniform01(n, stream=10 + 100 * rank)
            self.b_host = workloads.uniform01(n, stream=11 + 100 * rank)
            self.sets = [(mk.MLIRArray(self.a_host), mk.MLIRArray(self.b_host), mk.zeros(be, "Float32", n))
                         for _ in range(self.SETS)]
            self.a, self.b, self.c = self.sets[0]
            self.cursor = 0
            self.units_per_step = 12.0 * n
            self.h2d_bytes, self.d2h_bytes = 8 * n, 4 * n

        def launch(self):
            a, b, c = self.sets[self.cursor % self.SETS]
            self.cursor += 1
            _lib.check(L.mk_vadd_f32(c.pointer(), a.pointer(), b.pointer(), self.n, stream()), "vadd")

        def combine(self):
            pass

        def check(self):
            want = self.a_host + self.b_host
            for i, (_, _, c) in enumerate(self.sets[:min(self.cursor, self.SETS)]):
                if not np.array_equal(mk.Array(c), want):
                    raise CheckFailed(f"vadd: rank {rank} set {i} differs from a+b")

        def graph_breakdown(self, K):
            """CUDA-graph timing of K back-to-back launches over the rotating
            sets: the vadd with programmatic dependent launch (the product
            path), the same kernel launched plainly, and an empty kernel."""
            st = torch.zeros(2, dtype=torch.int64, device="cuda")
            res = {}
            for label, fn in (
                    ("graph_vadd_pdl", lambda a, b, c: L.mk_vadd_f32(c.pointer(), a.pointer(), b.pointer(), self.n,
                                                                     stream())),
                    ("graph_vadd_plain", lambda a, b, c: L.mk_probe_vadd_f32(2, c.pointer(), a.pointer(),
                                                                             b.pointer(), self.n, None, stream())),
                    ("graph_empty_kernel", lambda a, b, c: L.mk_probe_vadd_f32(0, c.pointer(), a.pointer(),
                                                                               b.pointer(), self.n, st.data_ptr(),
                                                                               stream()))):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    for i in range(K):
                        _lib.check(fn(*self.sets[i % self.SETS]), label)
                g.replay()
                torch.cuda.synchronize()
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                g.replay()
                e1.record()
                torch.cuda.synchronize()
                res[label] = {"per_launch_us": round(e0.elapsed_time(e1) * 1e3 / K, 2)}
                del g
            return res

        def extra_roofline(self, K, kern_ms):
            """Where a 12 MiB vadd's time goes (mk_probe_vadd_f32), launched
            exactly like the timed loop (L2 flush, event, launch, event; no
            synchronisation until the end): CUDA-event time and device-clock
            span (first block start to last block end) of an empty kernel with
            the same grid, a read-only pass over a and b, the vadd itself with
            and without the L2 flush, and a bulk-copy (cp.async.bulk) vadd;
            medians over K launches."""
            flush = torch.ones(256 * 2**20 // 4, dtype=torch.float32, device="cuda")
            scratch = mk.zeros(be, "Float32", self.n)
            R = K + 3
            out = {}
            for label, mode, do_flush in (("empty_kernel", 0, True), ("empty_kernel_no_flush", 0, False),
                                          ("read_a_b_only", 1, True), ("vadd", 2, True),
                                          ("vadd_l2_resident", 2, False), ("vadd_bulk_copy", 3, True)):
                st = torch.zeros((R, 2), dtype=torch.int64, device="cuda")
                st[:, 0] = -1  # all ones: no block start seen yet
                dst = scratch if mode == 1 else self.c
                evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(R)]
                torch.cuda.synchronize()
                for i in range(R):
                    if do_flush:
                        flush.sum()
                    evs[i][0].record()
                    _lib.check(L.mk_probe_vadd_f32(mode, dst.pointer(), self.a.pointer(), self.b.pointer(), self.n,
                                                   st[i].data_ptr(), stream()), "probe")
                    evs[i][1].record()
                torch.cuda.synchronize()
                t = st.cpu().numpy().view(np.uint64)
                ev = [evs[i][0].elapsed_time(evs[i][1]) * 1e3 for i in range(3, R)]
                span = [float(t[i, 1] - t[i, 0]) * 1e-3 for i in range(3, R)]
                out[label] = {"event_us": round(statistics.median(ev), 2),
                              "device_span_us": round(statistics.median(span), 2)}
                if mode in (2, 3) and not np.array_equal(mk.Array(self.c), self.a_host + self.b_host):
                    raise CheckFailed(f"vadd probe mode {mode}: c differs from a+b")
            out.update(self.graph_breakdown(K))
            return {"breakdown": out}

        def e2e_setup(self):
            self.pa = torch.from_numpy(self.a_host).pin_memory()
            self.pb = torch.from_numpy(self.b_host).pin_memory()
            self.pc = torch.empty(self.n, dtype=torch.float32).pin_memory()
            self.k = mk.vadd(be, 256)

        def e2e_step(self):
            mk.copyto(be, self.a, self.pa)
            mk.copyto(be, self.b, self.pb)
            self.k(self.c, self.a, self.b, ndrange=self.n)
            mk.copyto(be, self.pc, self.c)
            torch.cuda.current_stream().synchronize()
            return None

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            c = np.empty_like(self.a_host)
            return lambda: Lo.mlirb_vadd_f32(c.ctypes.data, self.a_host.ctypes.data, self.b_host.ctypes.data,
                                             self.n, 256), self.units_per_step, "full n=2^20 vadd, W=256"

    class Gather(Workload):
        name = "gather"
        metric = "indirect gather HBM GB/s (algorithmic 12 B/elem)"
        cfg = workloads.CONFIGS["gather"]

        def __init__(self):
            super().__init__(rank, world)
            n, na = self.n, self.na = n_override or self.cfg["n"], self.cfg["na"]
            self.a_host = workloads.uniform01(na, stream=20)  # replicated on every rank
            self.idx_host = workloads.indices1(n, na, stream=21 + 100 * rank)
            self.a, self.idx = mk.MLIRArray(self.a_host), mk.MLIRArray(self.idx_host)
            self.c = mk.zeros(be, "Float32", n)
            self.units_per_step = 12.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 4 * n

        def launch(self):
            _lib.check(L.mk_gather_f32(self.c.pointer(), self.a.pointer(), self.na, self.idx.pointer(), self.n,
                                       stream()), "gather")

        def combine(self):
            pass

        def check(self):
            got = mk.Array(self.c)
            if not np.array_equal(got, self.a_host[self.idx_host.astype(np.int64) - 1]):
                raise CheckFailed(f"gather: rank {rank} differs from a[idx]")

        def extra_roofline(self, K, kern_ms):
            """This GPU's random-read ceiling for the same array and count:
            mk_probe_random_read_f32 (no index or output stream), timed like
            the kernel.  The gather's time over the probe's is its fraction of
            what random 4-byte reads of `a` allow."""
            sums = torch.empty(dev_sms() * 8, dtype=torch.int32, device="cuda")
            ev = [torch.cuda.Event(enable_timing=True) for _ in range(2 * K)]
            for _ in range(3):
                _lib.check(L.mk_probe_random_read_f32(sums.data_ptr(), sums.numel(), self.a.pointer(), self.na,
                                                      self.n, 7, stream()), "probe")
            for i in range(K):
                ev[2 * i].record()
                _lib.check(L.mk_probe_random_read_f32(sums.data_ptr(), sums.numel(), self.a.pointer(), self.na,
                                                      self.n, 7 + i, stream()), "probe")
                ev[2 * i + 1].record()
            torch.cuda.synchronize()
            probe_ms = _dist_allreduce_max(sum(ev[2 * i].elapsed_time(ev[2 * i + 1]) for i in range(K)) / K)
            return {"random_ceiling": {
                "probe": "mk_probe_random_read_f32: n random 4-byte .cg reads of the same 2^27-float array, "
                         "no index/output streams",
                "probe_ms": round(probe_ms, 5),
                "reads_per_s": round(self.n / (probe_ms * 1e-3), 1),
                "gather_equiv_gbs": round(12.0 * self.n / (probe_ms * 1e-3) / 1e9, 1),
                "frac": round(probe_ms / kern_ms, 4)}}

        def e2e_setup(self):
            self.pidx = torch.from_numpy(self.idx_host).pin_memory()
            self.pc = torch.empty(self.n, dtype=torch.float32).pin_memory()
            self.k = mk.gather(be, 256)

        def e2e_step(self):
            mk.copyto(be, self.idx, self.pidx)
            self.k(self.c, self.a, self.idx, ndrange=self.n)
            mk.copyto(be, self.pc, self.c)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            c = np.empty(self.n, dtype=np.float32)
            return lambda: Lo.mlirb_gather_f32(c.ctypes.data, self.a_host.ctypes.data, self.na,
                                               self.idx_host.ctypes.data, self.n, 256), \
                self.units_per_step, "full 2^27 gather, W=256"

    class GatherCeiling(Workload):
        name = "gather_ceiling"
        metric = "random 4-byte reads of a 512 MiB array, GB/s (4 B per read)"
        cfg = workloads.CONFIGS["gather"]

        def __init__(self):
            super().__init__(rank, world)
            self.n, self.na = n_override or self.cfg["n"], self.cfg["na"]
            self.a_host = workloads.uniform01(self.na, stream=20)
            self.a = mk.MLIRArray(self.a_host)
            self.sums = torch.empty(dev_sms() * 8, dtype=torch.int32, device="cuda")
            self.units_per_step = 4.0 * self.n
            self.h2d_bytes, self.d2h_bytes = 0, 4 * self.sums.numel()

        def launch(self):
            _lib.check(L.mk_probe_random_read_f32(self.sums.data_ptr(), self.sums.numel(), self.a.pointer(),
                                                  self.na, self.n, 7, stream()), "probe")

        def combine(self):
            pass

        def check(self):
            # XOR of every word read, recomputed on the host with the same hash
            i = np.arange(self.n, dtype=np.uint64)
            h = (i.astype(np.uint32) ^ np.uint32(7)).astype(np.uint64)
            for sh, mul in ((16, 0x85EBCA6B), (13, 0xC2B2AE35), (16, None)):
                h ^= h >> np.uint64(sh)
                if mul is not None:
                    h = (h * np.uint64(mul)) & np.uint64(0xFFFFFFFF)
            pos = (h * np.uint64(self.na)) >> np.uint64(32)
            want = np.bitwise_xor.reduce(self.a_host.view(np.uint32)[pos])
            got = np.bitwise_xor.reduce(self.sums.cpu().numpy().view(np.uint32))
            if got != want:
                raise CheckFailed(f"gather_ceiling: XOR {got:#x}, host {want:#x}")

        def e2e_setup(self):
            pass

        def e2e_step(self):
            self.launch()
            return self.sums.cpu()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            c = np.empty(self.n, dtype=np.float32)
            idx = workloads.indices1(self.n, self.na, stream=21)
            return lambda: Lo.mlirb_gather_f32(c.ctypes.data, self.a_host.ctypes.data, self.na,
                                               idx.ctypes.data, self.n, 256), \
                4.0 * self.n, "the 2^27 CPU gather's random reads (4 B per read), W=256"

    class Scan(Workload):
        name = "scan"
        metric = "accumulate!(+) / cumsum HBM GB/s (8 B/element)"
        cfg = {"n": 1 << 28}

        def __init__(self):
            super().__init__(rank, world)
            n = self.n = n_override or self.cfg["n"]
            self.x_host = workloads.uniform01(n, stream=50 + 100 * rank)
            self.x = mk.MLIRArray(self.x_host)
            self.y = mk.zeros(be, "Float32", n)
            self.units_per_step = 8.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 4 * n

        def launch(self):
            _lib.check(L.mk_accumulate_f32(self.y.pointer(), self.x.pointer(), self.n, 0, 0.0, 0, stream()), "scan")

        def combine(self):
            pass

        def check(self):
            got = float(self.y.storage[-1].item())
            want = float(np.sum(self.x_host, dtype=np.float64))
            assert abs(got - want) <= 1e-6 * want, (got, want)

        def e2e_setup(self):
            self.px = torch.from_numpy(self.x_host).pin_memory()
            self.py = torch.empty(self.n, dtype=torch.float32).pin_memory()

        def e2e_step(self):
            mk.copyto(be, self.x, self.px)
            mk.accumulate(operator.add, self.y, self.x)
            mk.copyto(be, self.py, self.y)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            out = np.empty(self.n, dtype=np.float32)
            tot = np.empty(self.n // 512 + 2, dtype=np.float32)
            return lambda: Lo.mlirb_cumsum_f32(out.ctypes.data, self.x_host.ctypes.data, self.n, 256, tot.ctypes.data), \
                self.units_per_step, "full 2^28 cumsum: per-block fp32 scans + block-prefix pass, W=256"

    class Dims(Workload):
        name = "reduce_dims"
        metric = "sum(m; dims=1) HBM GB/s (4 B/element)"
        cfg = {"n": 1 << 14}

        def __init__(self):
            super().__init__(rank, world)
            r = self.r = n_override or self.cfg["n"]
            self.c = r
            self.m_host = workloads.uniform01(r * r, stream=60 + 100 * rank)
            self.m = mk.MLIRArray(self.m_host.reshape((r, r), order="F"))
            self.out = mk.zeros(be, "Float32", (1, r))
            self.units_per_step = 4.0 * r * r
            self.h2d_bytes, self.d2h_bytes = 4 * r * r, 4 * r

        def launch(self):
            _lib.check(L.mk_mapreduce_dim_f32(self.out.pointer(), self.m.pointer(), 1, self.r, self.c, 0, 0, 0.0,
                                              stream()), "dims")

        def combine(self):
            pass

        def check(self):
            got = mk.Array(self.out).ravel()[:8]
            want = self.m_host.reshape((self.r, self.c), order="F")[:, :8].astype(np.float64).sum(0)
            np.testing.assert_allclose(got, want, rtol=1e-5)

        def e2e_setup(self):
            self.pm = torch.from_numpy(self.m_host).pin_memory()
            self.po = torch.empty(self.c, dtype=torch.float32).pin_memory()

        def e2e_step(self):
            mk.copyto(be, self.m, self.pm)
            mk.reductions.mapreduce_dims_into(mk.identity, operator.add, self.out, self.m, 1)
            mk.copyto(be, self.po, self.out)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            out = np.empty(self.c, dtype=np.float32)
            return lambda: Lo.mlirb_sum_dims1_f32(out.ctypes.data, self.m_host.ctypes.data, self.r, self.c), \
                self.units_per_step, "full 16384x16384 sum(m; dims=1), OpenMP over columns"

    class Histogram(Workload):
        name = "histogram"
        metric = "histogram HBM GB/s (4 B/key)"
        cfg = workloads.CONFIGS["histogram"]
        launches_per_step = 1
        graph_steps = True     # zero the counts + histogram, K times, as one CUDA graph
        kernel_events = True

        def __init__(self):
            super().__init__(rank, world)
            n, nb = self.n, self.nb = n_override or self.cfg["n"], self.cfg["nbins"]
            self.keys_host = workloads.zipf_keys(n, nb, self.cfg["s"], stream=30 + 100 * rank)
            self.keys = mk.MLIRArray(self.keys_host)
            self.counts = mk.zeros(be, "UInt32", nb)
            self.peer = distributed.shared_peer() if world > 1 else None
            self.gouts = [torch.empty(nb, dtype=torch.int32, device="cuda") for _ in range(2)]
            self.step_no = 0
            self.units_per_step = 4.0 * n
            self.h2d_bytes, self.d2h_bytes = 4 * n, 4 * nb

        def prepare(self):
            self.counts.storage.zero_()  # bins accumulate: every step starts from zero

        def launch(self):
            if self.peer is not None:
                # fused and pipelined: local counts, then this rank's counts
                # published to every rank over NVLink and the previous step's
                # global counts folded, in the same launch
                self.step_no += 1
                _lib.check(L.mk_hist_u32_allreduce_async(self.gouts[self.step_no % 2].data_ptr(),
                                                         self.counts.pointer(), self.nb, self.keys.pointer(), self.n,
                                                         stream()), "hist allreduce")
            else:
                _lib.check(L.mk_hist_u32(self.counts.pointer(), self.nb, self.keys.pointer(), self.n, stream()),
                           "hist")

        def combine(self):
            pass  # N>1: the exchange is inside the kernel

        def finish(self):
            if self.peer is not None:
                _lib.check(L.mk_hist_allreduce_complete(stream()), "hist complete")

        def result(self):
            if self.peer is None:
                return mk.Array(self.counts)
            return self.gouts[self.step_no % 2].cpu().numpy().view(np.uint32)

        def check(self):
            # every N: the combined counts equal the oracle's counts of all
            # ranks' keys, summed mod 2^32 (u32 wrap-around)
            import oracle
            mine = oracle.hist(self.keys_host, self.nb)[0].astype(np.int64)
            want = (_dist_sum_i64(mine) % (1 << 32)).astype(np.uint32)
            got = self.result()
            if not np.array_equal(got, want):
                bad = int(np.flatnonzero(got != want)[0])
                raise CheckFailed(f"histogram: rank {rank} bin {bad + 1} has {got[bad]}, oracle {want[bad]}")

        def e2e_setup(self):
            self.pk = torch.from_numpy(self.keys_host).pin_memory()
            self.pc = torch.empty(self.nb, dtype=torch.int32).pin_memory()
            self.k = mk.histogram(be, 256)

        def e2e_step(self):
            mk.copyto(be, self.keys, self.pk)
            self.counts.storage.zero_()
            if self.peer is not None:
                self.peer.histogram(self.counts, self.keys, self.gouts[0])
                self.pc.copy_(self.gouts[0], non_blocking=True)
            else:
                self.k(self.counts, self.keys, ndrange=self.n)
                self.pc.copy_(self.counts.storage, non_blocking=True)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            counts = np.zeros(self.nb, dtype=np.uint32)
            return lambda: Lo.mlirb_hist_u32(counts.ctypes.data, self.nb, self.keys_host.ctypes.data, self.n, 256), \
                4.0 * self.n, "all 2^26 Zipf keys, per-lane atomics, W=256"

    class MatmulSimt(Workload):
        name = "matmul_simt"
        metric = "matmul C=A*B TFLOP/s (16x16 SIMT kernel)"
        unit = "TFLOP/s"
        cfg = workloads.CONFIGS["matmul"]

        def __init__(self):
            super().__init__(rank, world)
            m, n, k = self.m, self.nn, self.k = ((n_override,) * 3 if n_override
                                                 else (self.cfg["m"], self.cfg["n"], self.cfg["k"]))
            self.A_host = workloads.normal((m, k), stream=40 + 100 * rank)
            self.B_host = workloads.normal((k, n), stream=41)
            self.A, self.B = mk.MLIRArray(self.A_host), mk.MLIRArray(self.B_host)
            self.C = mk.zeros(be, "Float32", (m, n))
            self.units_per_step = 2.0 * m * n * k
            self.h2d_bytes, self.d2h_bytes = 4 * (m * k + k * n), 4 * m * n

        def launch(self):
            _lib.check(L.mk_matmul_tiled16_f32(self.C.pointer(), self.A.pointer(), self.B.pointer(), self.m, self.nn,
                                               self.k, self.m, self.k, self.m, stream()), "tiled16")

        def combine(self):
            pass

        def check(self):
            import oracle
            ii = np.array([0, 1, self.m // 2, self.m - 1]); jj = np.array([0, self.nn - 1, 17, self.nn // 2])
            got = mk.Array(self.C)[ii, jj]
            want = oracle.matmul_entries_f64(self.A_host, self.B_host, ii, jj)
            np.testing.assert_allclose(got, want, rtol=1e-4, atol=1e-3)

        def e2e_setup(self):
            self.pA = torch.from_numpy(self.A_host.ravel(order="F")).pin_memory()
            self.pB = torch.from_numpy(self.B_host.ravel(order="F")).pin_memory()
            self.pC = torch.empty(self.m * self.nn, dtype=torch.float32).pin_memory()
            self.kern = mk.mm_tiled_simt(be, (16, 16))

        def e2e_step(self):
            mk.copyto(be, self.A, self.pA)
            mk.copyto(be, self.B, self.pB)
            self.kern(self.C, self.A, self.B, ndrange=(self.m, self.nn))
            mk.copyto(be, self.pC, self.C)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            Cs = np.zeros((self.m, self.nn), dtype=np.float32, order="F")
            cols = 512
            return lambda: Lo.mlirb_mm_tiled16_f32(Cs.ctypes.data, self.A_host.ctypes.data, self.B_host.ctypes.data,
                                                   self.m, self.nn, self.k, self.m, self.k, self.m, 0, cols), \
                2.0 * self.m * cols * self.k, f"C[:, 1:{cols}] of the 8192^3 product (restated 16x16 tiles)"

    class Matmul(Workload):
        name = "matmul"
        metric = "matmul C=A*B TFLOP/s"
        launches_per_step = 3  # split_a, split_b, sgemm_tf32x3
        unit = "TFLOP/s"
        cfg = workloads.CONFIGS["matmul"]

        def __init__(self):
            super().__init__(rank, world)
            m, n, k = self.m, self.nn, self.k = ((n_override,) * 3 if n_override
                                                 else (self.cfg["m"], self.cfg["n"], self.cfg["k"]))
            self.A_host = workloads.normal((m, k), stream=40 + 100 * rank)
            self.B_host = workloads.normal((k, n), stream=41)
            self.A, self.B = mk.MLIRArray(self.A_host), mk.MLIRArray(self.B_host)
            self.C = mk.zeros(be, "Float32", (m, n))
            self.units_per_step = 2.0 * m * n * k
            self.h2d_bytes, self.d2h_bytes = 4 * (m * k + k * n), 4 * m * n

        def launch(self):
            _lib.check(L.mk_sgemm_3xtf32(self.C.pointer(), self.A.pointer(), self.B.pointer(), self.m, self.nn,
                                               self.k, self.m, self.k, self.m, stream()), "sgemm")

        def combine(self):
            pass

        def check(self):
            # this rank's row block: C*v against A*(B*v) in fp64 (rel 1e-5, the
            # configuration's tolerance) and sampled entries against fp64 dots
            import oracle
            Cm = mk.Array(self.C)
            v = np.random.Generator(np.random.Philox(9 + rank)).standard_normal(self.nn)
            want = oracle.matvec_chain_f64(self.A_host, self.B_host, v)
            err = np.linalg.norm(oracle.matvec_f64(Cm, v) - want) / np.linalg.norm(want)
            if not err <= 1e-5:
                raise CheckFailed(f"matmul: rank {rank} rel error of C*v {err:.3e} > 1e-5")
            ii = np.array([0, 1, self.m // 2, self.m - 1]); jj = np.array([0, self.nn - 1, 17, self.nn // 2])
            got = Cm[ii, jj]
            want = oracle.matmul_entries_f64(self.A_host, self.B_host, ii, jj)
            if not np.allclose(got, want, rtol=1e-4, atol=2e-4):
                raise CheckFailed(f"matmul: rank {rank} sampled entries {got} vs {want}")

        def e2e_setup(self):
            self.pA = torch.from_numpy(self.A_host.ravel(order="F")).pin_memory()
            self.pB = torch.from_numpy(self.B_host.ravel(order="F")).pin_memory()
            self.pC = torch.empty(self.m * self.nn, dtype=torch.float32).pin_memory()
            self.kern = mk.mm_tiled(be, (16, 16))

        def e2e_step(self):
            mk.copyto(be, self.A, self.pA)
            mk.copyto(be, self.B, self.pB)
            self.kern(self.C, self.A, self.B, ndrange=(self.m, self.nn))
            mk.copyto(be, self.pC, self.C)
            torch.cuda.current_stream().synchronize()

        def cpu_sample(self, threads):
            import oracle
            Lo = oracle.lib()
            Cs = np.zeros((self.m, self.nn), dtype=np.float32, order="F")
            cols = 512
            return lambda: Lo.mlirb_mm_tiled16_f32(Cs.ctypes.data, self.A_host.ctypes.data, self.B_host.ctypes.data,
                                                   self.m, self.nn, self.k, self.m, self.k, self.m, 0, cols), \
                2.0 * self.m * cols * self.k, f"C[:, 1:{cols}] of the 8192^3 product (restated 16x16 tiles)"

    table = {"reduce": Reduce, "maximum": Maximum, "findmax": FindMax, "vadd": Vadd, "gather": Gather,
             "gather_ceiling": GatherCeiling,
             "histogram": Histogram,
             "matmul": Matmul, "matmul_simt": MatmulSimt,
             "scan": Scan, "reduce_dims": Dims}
    return table[kind]()


# ---------------------------------------------------------------- runner ---

def time_cpu(fn, budget_s: float = 10.0, max_reps: int = 20) -> tuple[float, int]:
    fn()  # warm-up (page faults, thread pool)
    times = []
    t_end = time.perf_counter() + budget_s
    while len(times) < max_reps and (not times or time.perf_counter() < t_end):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def run_ours(kind: str, args, rank: int, world: int, local_rank: int) -> dict | None:
    import torch

    dev = torch.device("cuda", local_rank)
    torch.cuda.set_device(dev)
    w = make_workload(kind, rank, world, args.n)
    s = torch.cuda.current_stream()
    if getattr(w, "graph_steps", False):
        step_ms, kern_avg_max, clock_info = time_graph_steps(w, args, rank, dev, local_rank)
    else:
        step_ms, kern_avg_max, clock_info = time_eager_steps(w, args, rank, dev, local_rank)
    return finish_line(w, kind, args, rank, world, dev, s, step_ms, kern_avg_max, clock_info)


def hide_host_latency(us: float = 200.0) -> None:
    """Queue a ~200 us device spin before the start event, so that the GPU is
    still busy while the host enqueues the timed work: the region then holds
    device time only, not the host's launch latency after an idle GPU.  With
    N>1 a device-side barrier follows the spin (a blocking fused exchange of
    zero elements through the peer mailbox), so every rank's region starts
    when all GPUs are there, not at each host's own moment after the host
    barrier."""
    import torch
    import torch.distributed as dist
    multi = dist.is_initialized() and dist.get_world_size() > 1
    if multi:
        from cutilecpu_b200 import _lib, distributed
        distributed.shared_peer()  # created at start-up; never inside the spin (its set-up synchronises)
        out = torch.empty(1, dtype=torch.float64, device="cuda")
    torch.cuda._sleep(int(us * 1e-6 * 1.965e9))
    if multi:
        _lib.check(_lib.lib().mk_mapreduce_f32_allreduce(out.data_ptr(), None, 0, 0, 0, 0.0,
                                                          torch.cuda.current_stream().cuda_stream), "device barrier")


def time_eager_steps(w, args, rank: int, dev, local_rank: int):
    """K steps launched one by one, each kernel bracketed by CUDA events."""
    import torch

    from cutilecpu_b200 import distributed
    # L2 flush between launches: READ a 256 MiB buffer (2x L2), so the lines
    # it leaves behind are clean and the next launch pays no write-backs
    flush = torch.ones(256 * 2**20 // 4, dtype=torch.float32, device=dev) if w.needs_l2_flush else None
    s = torch.cuda.current_stream()

    def step():
        w.prepare()
        w.launch()
        w.combine()

    finish = getattr(w, "finish", lambda: None)

    # correctness of the benchmarked configuration, before timing
    step()
    finish()
    torch.cuda.synchronize()
    w.check()

    for _ in range(args.warmup):
        if flush is not None:
            flush_out = flush.sum()  # noqa: F841
        step()
    finish()
    torch.cuda.synchronize()
    distributed.barrier(device=dev)

    clocks = ClockSampler(local_rank).start() if rank == 0 else None
    K = args.steps
    k_start = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    k_end = [torch.cuda.Event(enable_timing=True) for _ in range(K)]
    torch.cuda.synchronize()
    distributed.barrier(device=dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    hide_host_latency()
    t0.record(s)
    for i in range(K):
        if flush is not None:
            flush_out = flush.sum()  # noqa: F841
        w.prepare()
        k_start[i].record(s)
        w.launch()
        k_end[i].record(s)
        w.combine()
    finish()
    t1.record(s)
    torch.cuda.synchronize()
    distributed.barrier(device=dev)
    clock_info = clocks.stop() if clocks is not None else None

    region_ms = t0.elapsed_time(t1)
    kern_ms = [a.elapsed_time(b) for a, b in zip(k_start, k_end)]
    kern_avg = sum(kern_ms) / K
    # whole-step time: the full region, or (with an L2 flush between steps)
    # the per-step kernel + combine time without the flush writes
    step_ms = region_ms / K if flush is None else kern_avg
    w.per_rank_ms = _dist_gather_f64(step_ms)
    step_ms = max(w.per_rank_ms)
    kern_avg_max = _dist_allreduce_max(kern_avg)
    return step_ms, kern_avg_max, clock_info


def time_graph_steps(w, args, rank: int, dev, local_rank: int):
    """K steps captured as one CUDA graph and replayed once inside the timed
    region, so no step pays a launch gap; the per-step time is the region over
    K.  Workloads with `kernel_events` also get a separate eager pass of K
    launches bracketed by CUDA events, for the kernel's own duration (the
    roofline); otherwise the kernel time is the step time."""
    import torch

    from cutilecpu_b200 import distributed
    s = torch.cuda.current_stream()
    finish = getattr(w, "finish", lambda: None)

    def step():
        w.prepare()
        w.launch()
        w.combine()

    step()  # first step, then its full check
    finish()
    torch.cuda.synchronize()
    w.check()
    for _ in range(args.warmup):
        step()
    finish()
    K = args.steps
    kern_avg = None
    if getattr(w, "kernel_events", False):
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(K)]
        torch.cuda.synchronize()
        distributed.barrier(device=dev)
        hide_host_latency()
        for i in range(K):
            w.prepare()
            ev[i][0].record(s)
            w.launch()
            ev[i][1].record(s)
            w.combine()
        finish()
        torch.cuda.synchronize()
        kern_avg = sum(a.elapsed_time(b) for a, b in ev) / K
    # capture on a dedicated stream that has run the steps once already: the
    # library's per-stream scratch is allocated on a stream's first use, which
    # cannot happen during capture
    cap = torch.cuda.Stream()
    cap.wait_stream(s)
    with torch.cuda.stream(cap):
        step()
        finish()
    s.wait_stream(cap)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=cap):
        for _ in range(K):
            step()
        finish()
    g.replay()  # the graph's own first replay (upload), untimed
    torch.cuda.synchronize()
    w.check()
    distributed.barrier(device=dev)
    clocks = ClockSampler(local_rank).start() if rank == 0 else None
    torch.cuda.synchronize()
    distributed.barrier(device=dev)
    t0 = torch.cuda.Event(enable_timing=True)
    t1 = torch.cuda.Event(enable_timing=True)
    hide_host_latency()
    t0.record(s)
    g.replay()
    t1.record(s)
    torch.cuda.synchronize()
    distributed.barrier(device=dev)
    clock_info = clocks.stop() if clocks is not None else None
    w.check()  # the timed replay's results too
    per_rank = _dist_gather_f64(t0.elapsed_time(t1) / K)
    del g
    w.per_rank_ms = per_rank
    step_ms = max(per_rank)
    kern_max = _dist_allreduce_max(kern_avg) if kern_avg is not None else step_ms
    return step_ms, kern_max, clock_info


def finish_line(w, kind: str, args, rank: int, world: int, dev, s, step_ms: float, kern_avg_max: float,
                clock_info) -> dict | None:
    """e2e, CPU baseline, roofline and the JSON line of one workload."""
    import torch

    from cutilecpu_b200 import distributed
    K = args.steps

    # end to end through the public API with pinned host buffers
    w.e2e_setup()
    Ke = max(1, min(K, args.e2e_steps))
    w.e2e_step()
    torch.cuda.synchronize()
    distributed.barrier(device=dev)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(s)
    for _ in range(Ke):
        w.e2e_step()
    e1.record(s)
    torch.cuda.synchronize()
    e2e_ms = _dist_allreduce_max(e0.elapsed_time(e1) / Ke)

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        import oracle
        oracle.lib().or_set_num_threads(host_threads())
        fn, units, sample = w.cpu_sample(oracle.num_threads())
        t, reps = time_cpu(fn, budget_s=args.cpu_budget)
        cpu = {"value": round(units / t / (1e12 if w.unit == "TFLOP/s" else 1e9), 3), "unit": w.unit,
               "cores": oracle.num_threads(), "kind": "port",
               "sample": f"{sample}; restated MLIRBackend (oracle/oracle.c), median of {reps} reps"}

    # collective on every rank (max over ranks), so before rank 0 goes on alone
    extra = w.extra_roofline(K, kern_avg_max) if hasattr(w, "extra_roofline") else {}
    if rank != 0:
        return None
    scale = 1e12 if w.unit == "TFLOP/s" else 1e9
    total_units = w.units_per_step * world
    peak, peak_kind = peaks()
    achieved = w.units_per_step / (kern_avg_max * 1e-3) / scale
    roof = None
    if w.unit == "GB/s":
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                "traffic": PROFILED_TRAFFIC.get(kind)}
    elif kind == "matmul":
        tp, tk = tensor_peak()
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": tp, "unit": "TFLOP/s",
                "frac": round(achieved / tp, 4), "peak_source": tk, "traffic": PROFILED_TRAFFIC.get(kind)}
    else:
        roof = {"bound": "simt-fp32", "achieved": round(achieved, 2), "peak": None, "unit": "TFLOP/s",
                "frac": None, "traffic": None}
    roof.update(extra)
    line = {
        "metric": w.metric, "value": round(total_units / (step_ms * 1e-3) / scale, 2), "unit": w.unit,
        "n_gpus": world, "steps": K, "warmup": args.warmup, "ms_per_step": round(step_ms, 5),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": w.dtype,
        "data": "synthetic (seeded numpy Philox, host-generated)",
        "config": config_of(kind, world, args.n),
        "impl_notes": IMPL_NOTES.get(kind),
        "e2e": {"value": round(total_units / (e2e_ms * 1e-3) / scale, 3), "unit": w.unit,
                "h2d_bytes_per_step": w.h2d_bytes, "d2h_bytes_per_step": w.d2h_bytes},
        "gpu_launches": K * w.launches_per_step,
        "roofline": roof,
        "kernel_ms": round(kern_avg_max, 5),
        "step_ms_per_rank": [round(v, 5) for v in getattr(w, "per_rank_ms", [])],
        "clocks": clock_info,
        "cpu_baseline": cpu,
    }
    return line


# dram__bytes_read.sum + dram__bytes_write.sum per launch of the dominant
# kernel at the benchmark's own size, from the one-pass ncu captures summarised
# in profiles/ (bytes).
PROFILED_TRAFFIC: dict[str, float | None] = {
    "reduce": 1073769216 + 3054848,       # mapreduce_kernel<abs2,+>, n = 2^28
    "vadd": 8398336 + 0,                  # vadd_f32_vec4, n = 2^20 (stores stay in L2)
    "gather": 14957786368 + 536444160,    # gather_f32_vec4 (.cg loads), n = 2^27
    "histogram": 268520960 + 5512192,     # hist_smem, n = 2^26
    "matmul": 5886670080 + 275036672,     # sgemm_tf32x3_pair, 8192^3 (split pre-pass excluded)
    "scan": 1074146816 + 1024940032,      # scan_kernel (look-back), n = 2^28
    "reduce_dims": 1073759744 + 3271168,  # seg_warp (16-byte loads), 16384 x 16384, dims=1
    "maximum": 1073788672 + 3324672,      # mapreduce_kernel<identity,max>, n = 2^28
    "findmax": 1073792000 + 3548928,      # findext_kernel<true>, n = 2^28
}


def host_threads() -> int:
    """All host threads this process may use (torchrun sets OMP_NUM_THREADS=1
    for its workers, so the OpenMP default is not trusted)."""
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference(kind: str, args, world: int = 1) -> dict:
    """The reference's CPU implementation of the path (restated MLIRBackend)."""
    import oracle

    from cutilecpu_b200 import workloads

    oracle.lib().or_set_num_threads(host_threads())
    threads = oracle.num_threads()
    cfg = workloads.CONFIGS
    L = oracle.lib()
    if kind == "reduce":
        n = cfg["reduce"]["n"]
        x = workloads.uniform_pm1(n, stream=1)
        tmp = np.empty(n + n // 512 + 2, dtype=np.float32)
        fn = lambda: L.mlirb_sum_sq_f32(x.ctypes.data, n, 256, tmp.ctypes.data)  # noqa: E731
        units, unit, metric = 4.0 * n, "GB/s", "mapreduce sum(x.^2) HBM GB/s"
        sample = "full 2^28-element sum(x.^2) per step"
    elif kind == "vadd":
        n = cfg["vadd"]["n"]
        a, b = workloads.uniform01(n, stream=10), workloads.uniform01(n, stream=11)
        c = np.empty_like(a)
        fn = lambda: L.mlirb_vadd_f32(c.ctypes.data, a.ctypes.data, b.ctypes.data, n, 256)  # noqa: E731
        units, unit, metric = 12.0 * n, "GB/s", "vadd HBM GB/s"
        sample = "full n=2^20 vadd per step"
    elif kind == "gather":
        n, na = cfg["gather"]["n"], cfg["gather"]["na"]
        a, idx = workloads.uniform01(na, stream=20), workloads.indices1(n, na, stream=21)
        c = np.empty(n, dtype=np.float32)
        fn = lambda: L.mlirb_gather_f32(c.ctypes.data, a.ctypes.data, na, idx.ctypes.data, n, 256)  # noqa: E731
        units, unit, metric = 12.0 * n, "GB/s", "indirect gather HBM GB/s (algorithmic 12 B/elem)"
        sample = "full 2^27 gather per step"
    elif kind == "histogram":
        n, nb = cfg["histogram"]["n"], cfg["histogram"]["nbins"]
        keys = workloads.zipf_keys(n, nb, 1.1, stream=30)
        counts = np.zeros(nb, dtype=np.uint32)
        fn = lambda: L.mlirb_hist_u32(counts.ctypes.data, nb, keys.ctypes.data, n, 256)  # noqa: E731
        units, unit, metric = 4.0 * n, "GB/s", "histogram HBM GB/s (4 B/key)"
        sample = "all 2^26 Zipf keys per step"
    elif kind == "scan":
        n = 1 << 28
        x = workloads.uniform01(n, stream=50)
        out = np.empty(n, dtype=np.float32)
        tot = np.empty(n // 512 + 2, dtype=np.float32)
        fn = lambda: L.mlirb_cumsum_f32(out.ctypes.data, x.ctypes.data, n, 256, tot.ctypes.data)  # noqa: E731
        units, unit, metric = 8.0 * n, "GB/s", "accumulate!(+) / cumsum HBM GB/s (8 B/element)"
        sample = "full 2^28 cumsum per step"
    elif kind == "reduce_dims":
        r = 1 << 14
        m = workloads.uniform01(r * r, stream=60)
        out = np.empty(r, dtype=np.float32)
        fn = lambda: L.mlirb_sum_dims1_f32(out.ctypes.data, m.ctypes.data, r, r)  # noqa: E731
        units, unit, metric = 4.0 * r * r, "GB/s", "sum(m; dims=1) HBM GB/s (4 B/element)"
        sample = "full 16384x16384 sum(m; dims=1) per step"
    elif kind in ("matmul", "matmul_simt"):
        m = cfg["matmul"]["m"]
        A = workloads.normal((m, m), stream=40)
        B = workloads.normal((m, m), stream=41)
        Cs = np.zeros((m, m), dtype=np.float32, order="F")
        cols = 512
        fn = lambda: L.mlirb_mm_tiled16_f32(Cs.ctypes.data, A.ctypes.data, B.ctypes.data, m, m, m, m, m, m,  # noqa
                                            0, cols)
        units, unit = 2.0 * m * cols * m, "TFLOP/s"
        metric = "matmul C=A*B TFLOP/s" + (" (16x16 SIMT kernel)" if kind == "matmul_simt" else "")
        sample = f"C[:, 1:{cols}] of the 8192^3 product per step"
    else:
        raise SystemExit(f"--impl reference: no CPU restatement of --kernel {kind}")
    for _ in range(args.warmup):
        fn()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        fn()
    dt = (time.perf_counter() - t0) / args.steps
    scale = 1e12 if unit == "TFLOP/s" else 1e9
    v = round(units / dt / scale, 3)
    return {"metric": metric, "value": v, "unit": unit, "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f32", "data": "synthetic (seeded numpy Philox, host-generated)", "impl": "reference",
            "config": config_of(kind, world, None),
            "cpu_baseline": {"value": v, "unit": unit, "cores": threads, "kind": "port",
                             "sample": sample + "; restated MLIRBackend (oracle/oracle.c); the Julia reference "
                                                "cannot run here (no julia)"},
            "e2e": {"value": v, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None)
    ap.add_argument("--warmup", type=int, default=None)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--kernel", default="baseline",
                    choices=["baseline", "reduce", "maximum", "findmax", "vadd", "gather", "gather_ceiling",
                             "histogram", "matmul", "matmul_simt", "scan", "reduce_dims", "all"],
                    help="baseline (default): the five BASELINE configurations, mapreduce last")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-budget", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--n", type=int, default=None,
                    help="override the element count of the configuration (small profiling cases)")
    args = ap.parse_args()
    if args.kernel == "baseline":
        kinds = list(BASELINE_KINDS)
    elif args.kernel == "all":
        kinds = ["maximum", "findmax", "gather_ceiling", "matmul_simt", "scan", "reduce_dims"] + BASELINE_KINDS
    else:
        kinds = [args.kernel]

    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local_rank = int(os.environ.get("LOCAL_RANK", "0"))

    if args.impl == "reference":
        if rank != 0:
            return
        if args.steps is None:
            args.steps = 5
        if args.warmup is None:
            args.warmup = 1
        for k in kinds:
            print(json.dumps(run_reference(k, args, world)), flush=True)
        return

    import torch
    import torch.distributed as dist
    if world > 1:
        torch.cuda.set_device(local_rank)
        dist.init_process_group("nccl", device_id=torch.device("cuda", local_rank))
        from cutilecpu_b200 import distributed
        distributed.shared_peer()  # the peer mailbox, set up once before any timing (collective)
        hide_host_latency(1.0)  # first device barrier: allocates its stream's reduction scratch now
        torch.cuda.synchronize()
    defaults = {"reduce": (2000, 50), "maximum": (1000, 20), "findmax": (1000, 20), "vadd": (2000, 50),
                "gather": (200, 10), "gather_ceiling": (200, 10), "histogram": (500, 20), "matmul": (20, 3),
                "matmul_simt": (3, 1), "scan": (500, 20), "reduce_dims": (1000, 20)}
    try:
        for k in kinds:
            a = argparse.Namespace(**vars(args))
            a.steps = args.steps if args.steps is not None else defaults[k][0]
            a.warmup = max(3, args.warmup if args.warmup is not None else defaults[k][1])
            try:
                line = run_ours(k, a, rank, world, local_rank)
            except CheckFailed as e:
                print(f"bench.py: result check failed: {e}", file=sys.stderr, flush=True)
                sys.exit(1)
            if line is not None:
                print(json.dumps(line), flush=True)
            gc.collect()
            torch.cuda.empty_cache()
    finally:
        if world > 1:
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
