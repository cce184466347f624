"""The KernelAbstractions launch surface: ``kernel(backend, wg)(args...; ndrange)``.

Python mirror of the reference's single launch choke point
``(obj::KA.Kernel{MLIRCUDABackend})(args...; ndrange, workgroupsize)``
(ext/MLIRCUDAExt.jl:540-548) and its set-up helpers ``_resolve_ndrange``
(:516-524), ``_resolve_wgsize`` (:477-497) and ``_launch_setup`` (:526-538),
with the same rules and error messages.  Where the reference JIT-compiles the
``@kernel`` body, each kernel here is one of the hot-path kernels of this
library, and a launch is one ``ccall``-equivalent into ``libkernels.so`` on
torch's current stream:

=================  =========================================  ===========================
kernel             reference definition                        C entry point
=================  =========================================  ===========================
``vadd``           test/test_gpu_simt.jl:13-16                 mk_vadd_f32
``gather``         ``c[i] = a[idx[i]]`` (src/lower.jl:4031)    mk_gather_f32
``histogram``      test/test_ka_cpu.jl:16-19, test_gpu_simt:49  mk_hist_u32
``mm_tiled``       examples/tiled_matmul.jl:28-48              mk_sgemm_3xtf32
``mm_naive``       examples/tiled_matmul.jl:12-19              mk_sgemm_f32
``mm_tiled_simt``  examples/tiled_matmul.jl:28-48 (SIMT)       mk_matmul_tiled16_f32
=================  =========================================  ===========================

The launch is asynchronous; ``synchronize(backend)`` waits and raises
``KernelException`` for device-flagged bad input, like CUDA.jl does.
"""
from __future__ import annotations

import math
from typing import Callable

from . import _lib
from .array import MLIRArray, MLIRCUDABackend, as_tuple, current_stream_handle, on_device


class KernelFunction:
    """A ``@kernel`` definition: calling it with a backend gives a ``Kernel``."""

    def __init__(self, name: str, rank: int, launcher: Callable, static_wg: tuple[int, ...] | None = None):
        self.name = name
        self.rank = rank            # ndrange rank the kernel indexes with
        self.launcher = launcher
        self.static_wg = static_wg  # workgroup the kernel body requires, if any

    def __call__(self, backend, workgroupsize=None, ndrange=None) -> "Kernel":
        if not isinstance(backend, MLIRCUDABackend):
            raise TypeError(f"{self.name}: backend must be MLIRCUDABackend, got {backend!r}")
        wg = as_tuple(workgroupsize) if workgroupsize is not None else None
        nd = as_tuple(ndrange) if ndrange is not None else None
        return Kernel(self, backend, wg, nd)

    def __repr__(self) -> str:
        return f"@kernel {self.name}"


class Kernel:
    """``KA.Kernel{MLIRCUDABackend}``: a kernel bound to the backend with an
    optional static workgroup size and ndrange."""

    def __init__(self, f: KernelFunction, backend, wg, nd):
        self.f, self.backend, self.wg, self.nd = f, backend, wg, nd

    def _resolve_ndrange(self, ndrange) -> tuple[int, ...]:
        if ndrange is not None:
            return as_tuple(ndrange)
        if self.nd is None:
            raise _lib.MLIRKernelsError(
                "MLIRCUDABackend: ndrange must be specified (kernel has no static ndrange)")
        return self.nd

    def _resolve_wgsize(self, workgroupsize, nd: tuple[int, ...]) -> tuple[int, ...]:
        if self.wg is not None:
            if workgroupsize is not None:
                wg = as_tuple(workgroupsize)
                if wg != self.wg:
                    raise _lib.MLIRKernelsError(
                        f"MLIRCUDABackend: workgroupsize={wg} conflicts with the kernel's "
                        f"static workgroupsize {self.wg}.")
            return self.wg
        if workgroupsize is None:
            return tuple(min(256, nd[0]) if d == 0 else 1 for d in range(len(nd)))
        return as_tuple(workgroupsize)

    def launch_setup(self, ndrange=None, workgroupsize=None):
        nd = self._resolve_ndrange(ndrange)
        wg = self._resolve_wgsize(workgroupsize, nd)
        if len(wg) != len(nd):
            raise _lib.MLIRKernelsError(
                f"MLIRCUDABackend: ndrange {nd} ({len(nd)}-D) and workgroupsize {wg} "
                f"({len(wg)}-D) must have the same number of dimensions.")
        if len(nd) != self.f.rank:
            raise _lib.MLIRKernelsError(
                f"MLIRCUDABackend: {self.f.name} indexes a {self.f.rank}-D ndrange, got {nd}")
        if any(w < 1 for w in wg) or math.prod(wg) > 1024:
            raise _lib.MLIRKernelsError(f"MLIRCUDABackend: invalid workgroupsize {wg}")
        if self.f.static_wg is not None and wg != self.f.static_wg:
            raise _lib.MLIRKernelsError(
                f"MLIRCUDABackend: {self.f.name} is written for workgroupsize {self.f.static_wg}, got {wg}")
        return nd, wg

    def __call__(self, *args, ndrange=None, workgroupsize=None):
        nd, wg = self.launch_setup(ndrange, workgroupsize)
        with on_device(*args):
            self.f.launcher(args, nd, wg, current_stream_handle())
        return None


def _need(a, name: str, eltypes: tuple[str, ...], min_len: int, what: str) -> MLIRArray:
    if not isinstance(a, MLIRArray):
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend: {what}: `{name}` must be an MLIRArray, got {type(a).__name__}")
    if a.eltype not in eltypes:
        raise _lib.MLIRKernelsError(
            f"MLIRCUDABackend: {what}: `{name}` has element type {a.eltype}, expected {' or '.join(eltypes)}")
    if a.length < min_len:
        raise _lib.MLIRKernelsError(
            f"MLIRCUDABackend: {what}: `{name}` has {a.length} elements, ndrange needs {min_len}")
    return a


# ---- launchers: argument checks + one C-ABI call each ----------------------

def _launch_vadd(args, nd, wg, stream) -> None:
    if len(args) != 3:
        raise _lib.MLIRKernelsError("vadd!(c, a, b): expected 3 arguments")
    n = nd[0]
    c = _need(args[0], "c", ("Float32",), n, "vadd!")
    a = _need(args[1], "a", ("Float32",), n, "vadd!")
    b = _need(args[2], "b", ("Float32",), n, "vadd!")
    _lib.check(_lib.lib().mk_vadd_f32(c.pointer(), a.pointer(), b.pointer(), n, stream), "vadd!")


def _launch_gather(args, nd, wg, stream) -> None:
    if len(args) != 3:
        raise _lib.MLIRKernelsError("gather!(c, a, idx): expected 3 arguments")
    n = nd[0]
    c = _need(args[0], "c", ("Float32",), n, "gather!")
    a = _need(args[1], "a", ("Float32",), 0, "gather!")
    idx = _need(args[2], "idx", ("Int32",), n, "gather!")
    _lib.check(_lib.lib().mk_gather_f32(c.pointer(), a.pointer(), a.length, idx.pointer(), n, stream),
               "gather!")


def _launch_histogram(args, nd, wg, stream) -> None:
    if len(args) != 2:
        raise _lib.MLIRKernelsError("histogram!(bins, keys): expected 2 arguments")
    n = nd[0]
    bins = _need(args[0], "bins", ("UInt32", "Int32", "Int64", "Float32"), 1, "histogram!")
    keys = _need(args[1], "keys", ("Int32", "Int64"), n, "histogram!")
    if bins.length > 2**31 - 1:
        raise _lib.MLIRKernelsError("histogram!: too many bins")
    bin_type = {"UInt32": 0, "Int32": 0, "Int64": 1, "Float32": 2}[bins.eltype]
    key_type = 0 if keys.eltype == "Int32" else 1
    _lib.check(_lib.lib().mk_hist(bins.pointer(), bin_type, bins.length, keys.pointer(), key_type, n, stream),
               "histogram!")


def _matmul_operands(args, nd, what):
    if len(args) != 3:
        raise _lib.MLIRKernelsError(f"{what}(C, A, B): expected 3 arguments")
    Cm, A, B = args
    for name, x in (("C", Cm), ("A", A), ("B", B)):
        _need(x, name, ("Float32",), 0, what)
        if x.ndims != 2:
            raise _lib.MLIRKernelsError(f"{what}: `{name}` must be a matrix, got dims {x.dims}")
    M, N = nd
    K = A.size(2)
    if A.size(1) < M or B.size(2) < N or B.size(1) < K or Cm.size(1) < M or Cm.size(2) < N:
        raise _lib.MLIRKernelsError(
            f"{what}: shapes C{Cm.dims} A{A.dims} B{B.dims} do not cover ndrange {nd}")
    return Cm, A, B, M, N, K


def _launch_mm_tiled(args, nd, wg, stream) -> None:
    Cm, A, B, M, N, K = _matmul_operands(args, nd, "mm_tiled!")
    _lib.check(_lib.lib().mk_sgemm_3xtf32(
        Cm.pointer(), A.pointer(), B.pointer(), M, N, K, A.size(1), B.size(1), Cm.size(1), stream),
        "mm_tiled!")


def _launch_mm_naive(args, nd, wg, stream) -> None:
    Cm, A, B, M, N, K = _matmul_operands(args, nd, "mm_naive!")
    _lib.check(_lib.lib().mk_sgemm_f32(
        Cm.pointer(), A.pointer(), B.pointer(), M, N, K, A.size(1), B.size(1), Cm.size(1), stream),
        "mm_naive!")


def mul(Cm: MLIRArray, A: MLIRArray, B: MLIRArray) -> MLIRArray:
    """``LinearAlgebra.mul!(C, A, B)`` on MLIRArrays: C = A*B over all K terms
    on the tcgen05 tensor cores (3xTF32)."""
    with on_device(Cm, A, B):
        _launch_mm_naive((Cm, A, B), (A.size(1), B.size(2)), None, current_stream_handle())
    return Cm


def _launch_mm_tiled_simt(args, nd, wg, stream) -> None:
    Cm, A, B, M, N, K = _matmul_operands(args, nd, "mm_tiled!")
    _lib.check(_lib.lib().mk_matmul_tiled16_f32(
        Cm.pointer(), A.pointer(), B.pointer(), M, N, K, A.size(1), B.size(1), Cm.size(1), stream),
        "mm_tiled!")


vadd = KernelFunction("vadd!", 1, _launch_vadd)
gather = KernelFunction("gather!", 1, _launch_gather)
histogram = KernelFunction("histogram!", 1, _launch_histogram)
# mm_naive! (one output per thread, all K terms; examples/tiled_matmul.jl:12-19).
mm_naive = KernelFunction("mm_naive!", 2, _launch_mm_naive)
# mm_tiled! on the tcgen05 tensor cores in 3xTF32 (the hot path).
mm_tiled = KernelFunction("mm_tiled!", 2, _launch_mm_tiled, static_wg=(16, 16))
# The reference's 16x16 @localmem kernel run on CUDA cores (SIMT comparison point).
mm_tiled_simt = KernelFunction("mm_tiled!", 2, _launch_mm_tiled_simt, static_wg=(16, 16))


class Scale:
    """The closure ``x -> a * x`` (a Float32 constant), for ``map_``."""

    def __init__(self, a: float):
        self.a = float(a)


def axpby(dst: MLIRArray, a: float, x: MLIRArray, b: float = 0.0, y: MLIRArray | None = None) -> MLIRArray:
    """``dst .= a .* x .+ b .* y`` (or ``a .* x`` without y), bit-exact with
    Julia's Float32 evaluation order."""
    n = x.length
    _need(dst, "dst", ("Float32",), n, "axpby")
    _need(x, "x", ("Float32",), n, "axpby")
    if y is not None:
        _need(y, "y", ("Float32",), n, "axpby")
    with on_device(dst, x, y):
        _lib.check(_lib.lib().mk_axpby_f32(dst.pointer(), a, x.pointer(), b, y.pointer() if y is not None else None,
                                           n, current_stream_handle()), "axpby")
    return dst


def map_(f, dst: MLIRArray, src: MLIRArray) -> MLIRArray:
    """``AK.map!(f, dst, src)`` for the closures this library implements:
    ``Scale(a)`` (x -> a*x)."""
    if isinstance(f, Scale):
        return axpby(dst, f.a, src)
    raise _lib.MLIRKernelsError(f"MLIRCUDABackend: map! has no kernel for {f!r} (supported: Scale(a))")
