"""Full reductions: the AcceleratedKernels / GPUArrays reduce surface.

Python mirror of ``GPUArrays.mapreducedim!`` (ext/MLIRCUDAExt.jl:100-121) and
of the AcceleratedKernels entry points the reference's tests call on an
MLIRArray (``AK.reduce``, ``AK.mapreduce``, ``AK.sum``, ``AK.count``;
test/test_downstream_ka.jl:26-35; Base ``sum``/``maximum``/``minimum``/``prod``/
``count``/``mapreduce`` of test/test_gpuarrays.jl:83-91).

Every call is ONE fused launch of ``mk_mapreduce_f32``: ``f`` is applied while
the data streams through (a ``Broadcasted`` argument such as ``x.^2`` is not
materialised, unlike :103 of the reference), and the partials are folded on the
device (no host copy of partials, unlike :125-131).  Sums and products
accumulate in fp64, so results are within rel 1e-5 of an fp64 reference; max
and min are exact.  The result is returned to the host as a Python number.
"""
from __future__ import annotations

import operator

import torch

from . import _lib
from .array import MLIRArray, current_stream_handle


def identity(x):
    return x


def abs2(x):
    """``abs2(x) = x*x`` (what ``x.^2`` maps each element to)."""
    return x * x


def positive(x):
    """The predicate ``>(0)``, i.e. ``x -> x > 0``."""
    return x > 0


_F = {identity: "identity", abs2: "abs2", abs: "abs", positive: "gt0"}
_OP = {operator.add: "add", max: "max", min: "min", operator.mul: "mul"}
_NEUTRAL = {"add": 0.0, "mul": 1.0, "max": float("-inf"), "min": float("inf")}


class Broadcasted:
    """A lazy ``f.(x)`` (Base.Broadcast.Broadcasted with one array argument).

    ``mapreduce(identity, +, Broadcasted(abs2, x))`` is ``sum(x.^2)`` and runs as
    a single fused pass."""

    def __init__(self, f, arg: MLIRArray):
        self.f, self.arg = f, arg


def _f_name(f) -> str:
    try:
        return _F[f]
    except (KeyError, TypeError):
        raise _lib.MLIRKernelsError(
            f"MLIRCUDABackend: mapreduce has no kernel for f={getattr(f, '__name__', f)!r} "
            "(supported: identity, abs2, abs, >(0))") from None


def _op_name(op) -> str:
    try:
        return _OP[op]
    except (KeyError, TypeError):
        raise _lib.MLIRKernelsError(
            f"MLIRCUDABackend: mapreduce has no kernel for op={getattr(op, '__name__', op)!r} "
            "(supported: +, *, max, min)") from None


def _unwrap(f, src):
    if isinstance(src, Broadcasted):
        if f is not identity:
            raise _lib.MLIRKernelsError("MLIRCUDABackend: mapreduce(f, op, f2.(x)) supports f = identity only")
        f, src = src.f, src.arg
    if not isinstance(src, MLIRArray):
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend: reduce source must be an MLIRArray, got {type(src).__name__}")
    if src.eltype != "Float32":
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend: reductions take Float32 sources, got {src.eltype}")
    return f, src


def mapreduce_device(f, op, src, init=None, out: torch.Tensor | None = None) -> torch.Tensor:
    """Launch the fused reduction and return the 1-element fp64 device tensor
    holding the result (asynchronous; no host synchronisation)."""
    f, src = _unwrap(f, src)
    fname, opname = _f_name(f), _op_name(op)
    init_v = _NEUTRAL[opname] if init is None else float(init)
    if out is None:
        out = torch.empty(1, dtype=torch.float64, device=src.storage.device)
    _lib.check(_lib.lib().mk_mapreduce_f32(out.data_ptr(), src.pointer(), src.length,
                                           _lib.MK_F[fname], _lib.MK_OP[opname], init_v,
                                           current_stream_handle()), "mapreduce")
    return out


def mapreduce(f, op, src, init=None, neutral=None):
    """``AK.mapreduce(f, op, src; init, neutral)`` / Base ``mapreduce``."""
    del neutral  # the kernel uses op's own identity element
    return mapreduce_device(f, op, src, init).item()


def reduce(op, src, init=None, neutral=None):
    """``AK.reduce(op, src; init)``."""
    return mapreduce(identity, op, src, init=init, neutral=neutral)


def sum(f_or_src, src=None):
    """``sum(x)`` or ``sum(f, x)``."""
    if src is None:
        return mapreduce(identity, operator.add, f_or_src)
    return mapreduce(f_or_src, operator.add, src)


def prod(src):
    return mapreduce(identity, operator.mul, src)


def maximum(src):
    return mapreduce(identity, max, src)


def minimum(src):
    return mapreduce(identity, min, src)


def count(pred, src) -> int:
    """``count(pred, x)``; ``pred`` must be ``positive`` (``>(0)``)."""
    if pred is not positive:
        raise _lib.MLIRKernelsError("MLIRCUDABackend: count supports the predicate >(0) only")
    return int(mapreduce(positive, operator.add, src))


def mapreducedim(f, op, R: MLIRArray, A, init=None) -> MLIRArray:
    """``GPUArrays.mapreducedim!(f, op, R, A; init)`` for a full reduction
    (``length(R) == 1``), the form ``sum``/``mapreduce`` reach: the result is
    written into ``R`` on the device, with no host round trip."""
    if R.length != 1:
        raise _lib.MLIRKernelsError(
            "MLIRCUDABackend.mapreducedim!: only full reductions (length(R) == 1) are supported")
    if R.eltype not in ("Float32", "Float64"):
        raise _lib.MLIRKernelsError(f"mapreducedim!: result eltype {R.eltype} unsupported")
    res = mapreduce_device(f, op, A, init)
    R.storage.copy_(res.to(R.storage.dtype))
    return R
