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

import math
import operator

import torch

from . import _lib
from .array import MLIRArray, current_stream_handle, on_device


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
    with on_device(src):
        _lib.check(_lib.lib().mk_mapreduce_f32(out.data_ptr(), src.pointer(), src.length,
                                               _lib.MK_F[fname], _lib.MK_OP[opname], init_v,
                                               current_stream_handle()), "mapreduce")
    return out


def mapreduce_dims_into(f, op, R: MLIRArray, A, dim: int, init=None) -> MLIRArray:
    """Reduce the 1-based dimension ``dim`` of ``A`` into ``R`` (Float32, same
    dims as ``A`` with ``size(R, dim) == 1``): one ``mk_mapreduce_dim_f32``."""
    f, A = _unwrap(f, A)
    fname, opname = _f_name(f), _op_name(op)
    if not 1 <= dim <= max(1, A.ndims):
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend: dims={dim} out of range for {A.dims}")
    if R.eltype != "Float32":
        raise _lib.MLIRKernelsError(f"mapreducedim!: dims result eltype {R.eltype} unsupported")
    pre = math.prod(A.dims[:dim - 1])
    ln = A.dims[dim - 1] if dim <= A.ndims else 1
    post = math.prod(A.dims[dim:])
    if R.length != pre * post:
        raise _lib.MLIRKernelsError(f"mapreducedim!: result dims {R.dims} do not match reducing {A.dims} over {dim}")
    init_v = _NEUTRAL[opname] if init is None else float(init)
    with on_device(R, A):
        _lib.check(_lib.lib().mk_mapreduce_dim_f32(R.pointer(), A.pointer(), pre, ln, post, _lib.MK_F[fname],
                                                   _lib.MK_OP[opname], init_v, current_stream_handle()),
                   "mapreducedim!")
    return R


def _dims_result(f, op, A, dims: int, init=None) -> MLIRArray:
    from .array import MLIRCUDABackend, allocate
    _, src = _unwrap(f, A)
    rdims = tuple(1 if d == dims - 1 else n for d, n in enumerate(src.dims))
    R = allocate(MLIRCUDABackend(), "Float32", rdims)
    return mapreduce_dims_into(f, op, R, A, dims, init)


def mapreduce(f, op, src, init=None, neutral=None, dims=None):
    """``AK.mapreduce(f, op, src; init, neutral, dims)`` / Base ``mapreduce``:
    a number, or with ``dims`` an MLIRArray with that dimension reduced."""
    del neutral  # the kernel uses op's own identity element
    if dims is not None:
        return _dims_result(f, op, src, dims, init)
    return mapreduce_device(f, op, src, init).item()


def reduce(op, src, init=None, neutral=None, dims=None):
    """``AK.reduce(op, src; init, dims)``."""
    return mapreduce(identity, op, src, init=init, neutral=neutral, dims=dims)


def sum(f_or_src, src=None, dims=None):
    """``sum(x)``, ``sum(f, x)`` or with ``dims=d``."""
    if src is None:
        return mapreduce(identity, operator.add, f_or_src, dims=dims)
    return mapreduce(f_or_src, operator.add, src, dims=dims)


def prod(src, dims=None):
    return mapreduce(identity, operator.mul, src, dims=dims)


def maximum(src, dims=None):
    return mapreduce(identity, max, src, dims=dims)


def minimum(src, dims=None):
    return mapreduce(identity, min, src, dims=dims)


def count(pred, src) -> int:
    """``count(pred, x)``; ``pred`` must be ``positive`` (``>(0)``)."""
    if pred is not positive:
        raise _lib.MLIRKernelsError("MLIRCUDABackend: count supports the predicate >(0) only")
    return int(mapreduce(positive, operator.add, src))


def mapreducedim(f, op, R: MLIRArray, A, init=None) -> MLIRArray:
    """``GPUArrays.mapreducedim!(f, op, R, A; init)``.  A full reduction
    (``length(R) == 1``) is one fused launch written into ``R`` on the device;
    otherwise exactly one dimension may be reduced (the reference allows only
    single-dim reductions too, ext/MLIRCUDAExt.jl:115-117)."""
    if R.eltype not in ("Float32", "Float64"):
        raise _lib.MLIRKernelsError(f"mapreducedim!: result eltype {R.eltype} unsupported")
    _, src = _unwrap(f, A)
    if R.length == 1 and src.length != 1:
        res = mapreduce_device(f, op, A, init)
        R.storage.copy_(res.to(R.storage.dtype))
        return R
    rd = tuple(d + 1 for d in range(src.ndims) if R.size(d + 1) == 1 and src.size(d + 1) != 1)
    if len(rd) != 1:
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend.mapreducedim!: only single-dim reductions (got dims={rd})")
    return mapreduce_dims_into(f, op, R, A, rd[0], init)


def accumulate(op, dst: MLIRArray, src: MLIRArray, init=None, inclusive: bool = True) -> MLIRArray:
    """``AK.accumulate!(op, dst, src; init, inclusive)``: prefix scan of a
    Float32 vector into ``dst`` (which may be ``src``) in one launch."""
    for name, a in (("dst", dst), ("src", src)):
        if not isinstance(a, MLIRArray) or a.eltype != "Float32":
            raise _lib.MLIRKernelsError(f"accumulate!: `{name}` must be a Float32 MLIRArray")
    if dst.length < src.length:
        raise _lib.MLIRKernelsError("accumulate!: dst is shorter than src")
    opname = _op_name(op)
    init_v = _NEUTRAL[opname] if init is None else float(init)
    with on_device(dst, src):
        _lib.check(_lib.lib().mk_accumulate_f32(dst.pointer(), src.pointer(), src.length, _lib.MK_OP[opname],
                                                init_v, 0 if inclusive else 1, current_stream_handle()),
                   "accumulate!")
    return dst


def cumsum(src: MLIRArray) -> MLIRArray:
    """``cumsum(x)`` / ``AK.cumsum(x)``: a new MLIRArray of running sums."""
    from .array import MLIRCUDABackend, allocate
    dst = allocate(MLIRCUDABackend(), "Float32", src.dims)
    return accumulate(operator.add, dst, src)


def _findext(src: MLIRArray, find_max: bool):
    if not isinstance(src, MLIRArray) or src.eltype != "Float32":
        raise _lib.MLIRKernelsError("findmax/findmin take a Float32 MLIRArray")
    if src.length == 0:
        raise ValueError("collection must be non-empty")
    val = torch.empty(1, dtype=torch.float64, device=src.storage.device)
    idx = torch.empty(1, dtype=torch.int64, device=src.storage.device)
    with on_device(src):
        _lib.check(_lib.lib().mk_findext_f32(val.data_ptr(), idx.data_ptr(), src.pointer(), src.length,
                                             int(find_max), current_stream_handle()), "findmax")
    return float(val.item()), int(idx.item())


def findmax(src: MLIRArray):
    """``findmax(x)``: (maximum, 1-based index of its first occurrence); NaN
    counts as the maximum, as in Julia."""
    return _findext(src, True)


def findmin(src: MLIRArray):
    """``findmin(x)``: (minimum, 1-based index); NaN counts as the minimum."""
    return _findext(src, False)


def argmax(src: MLIRArray) -> int:
    return findmax(src)[1]


def argmin(src: MLIRArray) -> int:
    return findmin(src)[1]


def extrema(src: MLIRArray):
    """``extrema(x)`` = (minimum(x), maximum(x))."""
    return minimum(src), maximum(src)


def any_(pred, src) -> bool:
    """``any(>(0), x)``."""
    return count(pred, src) > 0


def all_(pred, src) -> bool:
    """``all(>(0), x)``."""
    return count(pred, src) == src.length
