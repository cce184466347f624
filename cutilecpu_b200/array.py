"""MLIRArray and the KernelAbstractions backend protocol of MLIRCUDABackend.

Python mirror of ext/MLIRCUDAExt.jl:31-161: ``MLIRArray{T,N}`` (:50-68) is a
device array whose ``get_backend`` routes launches to this library;
``allocate``/``zeros``/``ones``/``synchronize``/``functional``/
``supports_atomics``/``copyto`` follow :139-147 and ``launch_config`` :154-161.

Storage is a flat torch CUDA tensor in Julia (column-major) element order, so a
``(M, N)`` MLIRArray has element ``(i, j)`` (1-based in Julia, 0-based here) at
offset ``i + j*M`` exactly like the ``CuArray`` the reference wraps.  Device
memory, streams and copies come from torch; every computation goes through
``libkernels.so``.
"""
from __future__ import annotations

import math
from typing import Iterable, Sequence

import numpy as np
import torch

from . import _lib

# Julia element type name -> (numpy dtype, torch storage dtype).  UInt32 is
# stored in an int32 tensor and reinterpreted bit-for-bit on the host.
ELTYPES = {
    "Float32": (np.dtype(np.float32), torch.float32),
    "Float64": (np.dtype(np.float64), torch.float64),
    "Int32": (np.dtype(np.int32), torch.int32),
    "UInt32": (np.dtype(np.uint32), torch.int32),
    "Int64": (np.dtype(np.int64), torch.int64),
}
_BY_NUMPY = {np.dtype(np.float32): "Float32", np.dtype(np.float64): "Float64",
             np.dtype(np.int32): "Int32", np.dtype(np.uint32): "UInt32",
             np.dtype(np.int64): "Int64"}
_BY_TORCH = {torch.float32: "Float32", torch.float64: "Float64", torch.int32: "Int32",
             torch.int64: "Int64"}


def eltype_name(T) -> str:
    """Normalise a Julia-style name, numpy dtype or torch dtype to a name."""
    if isinstance(T, str):
        if T not in ELTYPES:
            raise TypeError(f"MLIRCUDABackend: unsupported element type {T}")
        return T
    if isinstance(T, torch.dtype):
        if T not in _BY_TORCH:
            raise TypeError(f"MLIRCUDABackend: unsupported element type {T}")
        return _BY_TORCH[T]
    dt = np.dtype(T)
    if dt not in _BY_NUMPY:
        raise TypeError(f"MLIRCUDABackend: unsupported element type {dt}")
    return _BY_NUMPY[dt]


def _dims(dims) -> tuple[int, ...]:
    if isinstance(dims, (int, np.integer)):
        dims = (int(dims),)
    dims = tuple(int(d) for d in dims)
    if any(d < 0 for d in dims):
        raise ValueError(f"negative dimension in {dims}")
    return dims


class MLIRArray:
    """A device array in Julia layout whose backend is MLIRCUDABackend.

    ``MLIRArray(x)`` copies a host numpy array (any order; Julia dims = x.shape)
    or wraps a CUDA torch tensor without a copy when its memory is already in
    column-major order (a 1-D contiguous tensor always is).
    """

    __slots__ = ("storage", "dims", "eltype")

    def __init__(self, data, dims: Sequence[int] | None = None, eltype: str | None = None):
        if isinstance(data, torch.Tensor):
            if data.device.type != "cuda":
                raise ValueError("MLIRArray wraps CUDA tensors; copy host data with MLIRArray(numpy_array)")
            name = eltype or eltype_name(data.dtype)
            t = data
            jdims = _dims(dims) if dims is not None else tuple(t.shape)
            if t.dim() > 1 and dims is None:
                # Julia dims = torch shape; column-major storage
                t = t.permute(*reversed(range(t.dim())))
                if not t.is_contiguous():
                    t = t.contiguous()
            if not t.is_contiguous():
                t = t.contiguous()
            flat = t.reshape(-1)
            if flat.numel() != math.prod(jdims):
                raise ValueError(f"dims {jdims} do not match {flat.numel()} elements")
            self.storage, self.dims, self.eltype = flat, jdims, name
        else:
            arr = np.asarray(data)
            name = eltype or eltype_name(arr.dtype)
            npdt, tdt = ELTYPES[name]
            host = np.ascontiguousarray(arr.astype(npdt, copy=False).ravel(order="F"))
            if name == "UInt32":
                host = host.view(np.int32)
            self.storage = torch.from_numpy(host).to("cuda", non_blocking=False)
            if self.storage.dtype != tdt:
                self.storage = self.storage.to(tdt)
            self.dims, self.eltype = _dims(arr.shape), name

    # ---- Julia-style queries -------------------------------------------------
    @property
    def shape(self) -> tuple[int, ...]:
        return self.dims

    def size(self, d: int | None = None):
        """``size(a)`` or the 1-based ``size(a, d)``."""
        if d is None:
            return self.dims
        return self.dims[d - 1] if d <= len(self.dims) else 1

    def __len__(self) -> int:
        return math.prod(self.dims)

    @property
    def length(self) -> int:
        return math.prod(self.dims)

    @property
    def ndims(self) -> int:
        return len(self.dims)

    def strides(self) -> tuple[int, ...]:
        """Column-major strides in elements (``Base.strides``)."""
        s, out = 1, []
        for d in self.dims:
            out.append(s)
            s *= d
        return tuple(out)

    @property
    def device(self) -> int:
        return self.storage.device.index

    def pointer(self) -> int:
        """Device address of the first element (``Base.pointer``)."""
        return self.storage.data_ptr()

    def view(self, lo: int, hi: int) -> "MLIRArray":
        """``@view a[lo:hi]`` (1-based, inclusive): a 1-D MLIRArray sharing this
        array's storage, like GPUArrays' ``derive`` of a contiguous view."""
        if not 1 <= lo <= hi + 1 or hi > self.length:
            raise IndexError(f"view {lo}:{hi} out of bounds for {self.length} elements")
        return MLIRArray(self.storage[lo - 1:hi], dims=(hi - lo + 1,), eltype=self.eltype)

    def to_numpy(self) -> np.ndarray:
        """``Array(a)``: a host copy with Julia dims, Fortran order."""
        host = self.storage.detach().cpu().numpy()
        if self.eltype == "UInt32":
            host = host.view(np.uint32)
        return host.reshape(self.dims, order="F")

    def __repr__(self) -> str:
        return f"MLIRArray{{{self.eltype},{len(self.dims)}}}(dims={self.dims}, device=cuda:{self.device})"


def Array(a: MLIRArray) -> np.ndarray:
    """``Array(a)``: copy an MLIRArray to the host."""
    return a.to_numpy()


class MLIRCUDABackend:
    """KernelAbstractions backend of this library (ext/MLIRCUDAExt.jl:31)."""

    def __eq__(self, other) -> bool:
        return isinstance(other, MLIRCUDABackend)

    def __hash__(self) -> int:
        return hash(MLIRCUDABackend)

    def __repr__(self) -> str:
        return "MLIRCUDABackend()"


def get_backend(x) -> MLIRCUDABackend:
    """``KA.get_backend(::MLIRArray) = MLIRCUDABackend()`` (ext/MLIRCUDAExt.jl:139)."""
    if isinstance(x, MLIRArray):
        return MLIRCUDABackend()
    raise TypeError(f"get_backend: {type(x).__name__} is not an MLIRArray")


def _check_backend(backend) -> None:
    if not isinstance(backend, MLIRCUDABackend):
        raise TypeError(f"expected MLIRCUDABackend, got {backend!r}")


def allocate(backend, T, dims) -> MLIRArray:
    """``KA.allocate(::MLIRCUDABackend, T, dims)``: uninitialised device array."""
    _check_backend(backend)
    name = eltype_name(T)
    d = _dims(dims)
    t = torch.empty(math.prod(d), dtype=ELTYPES[name][1], device="cuda")
    return MLIRArray(t, dims=d, eltype=name)


def zeros(backend, T, dims) -> MLIRArray:
    a = allocate(backend, T, dims)
    a.storage.zero_()
    return a


def ones(backend, T, dims) -> MLIRArray:
    a = allocate(backend, T, dims)
    a.storage.fill_(1)
    return a


def functional(backend) -> bool:
    """CUDA usable and libkernels.so loadable (``KA.functional``)."""
    _check_backend(backend)
    if not torch.cuda.is_available():
        return False
    try:
        _lib.lib()
    except Exception:
        return False
    return True


def supports_atomics(backend) -> bool:
    _check_backend(backend)
    return True


def on_device(*arrays):
    """Context in which a launch on ``arrays`` happens: their device made
    current (the library launches on the current device and its current
    stream), after checking that they all live on the same device."""
    import contextlib
    devs = {a.device for a in arrays if isinstance(a, MLIRArray)}
    if len(devs) > 1:
        raise _lib.MLIRKernelsError(f"MLIRCUDABackend: arguments live on different devices {sorted(devs)}")
    if not devs or next(iter(devs)) == torch.cuda.current_device():
        return contextlib.nullcontext()
    return torch.cuda.device(next(iter(devs)))


def current_stream_handle() -> int:
    """cudaStream_t of torch's current stream (CUDA.jl's task-local stream)."""
    return torch.cuda.current_stream().cuda_stream


def synchronize(backend) -> None:
    """``KA.synchronize``: wait for the device, then raise KernelException if a
    kernel flagged bad input (CUDA.jl's exception check, ext/MLIRCUDAExt.jl:317-335)."""
    _check_backend(backend)
    torch.cuda.synchronize()
    _lib.check(_lib.lib().mk_error_poll(current_stream_handle()), "synchronize")


def copyto(backend, dst, src):
    """``KA.copyto!(backend, dst, src)``: host<->device or device<->device.

    A host side given as a pinned torch CPU tensor copies asynchronously on the
    current stream; a numpy array copies synchronously."""
    _check_backend(backend)
    if isinstance(dst, MLIRArray) and isinstance(src, torch.Tensor):
        # host tensor: asynchronous on the current stream when it is pinned
        if src.numel() != dst.length:
            raise ValueError("copyto!: size mismatch")
        dst.storage.copy_(src.reshape(-1), non_blocking=src.device.type == "cpu" and src.is_pinned())
    elif isinstance(dst, torch.Tensor) and isinstance(src, MLIRArray):
        if dst.numel() != src.length:
            raise ValueError("copyto!: size mismatch")
        dst.reshape(-1).copy_(src.storage, non_blocking=dst.device.type == "cpu" and dst.is_pinned())
    elif isinstance(dst, MLIRArray) and isinstance(src, MLIRArray):
        if dst.length != src.length or dst.eltype != src.eltype:
            raise ValueError("copyto!: size or element type mismatch")
        dst.storage.copy_(src.storage)
    elif isinstance(dst, MLIRArray):
        host = np.asarray(src).astype(ELTYPES[dst.eltype][0], copy=False).ravel(order="F")
        if host.size != dst.length:
            raise ValueError("copyto!: size mismatch")
        if dst.eltype == "UInt32":
            host = host.view(np.int32)
        dst.storage.copy_(torch.from_numpy(np.ascontiguousarray(host)))
    elif isinstance(src, MLIRArray):
        host = src.to_numpy()
        dst[...] = host.reshape(dst.shape, order="F")
    else:
        raise TypeError("copyto!: one side must be an MLIRArray")
    return dst


def launch_config(kernel, ndrange, workgroupsize):
    """``KA.launch_config`` (ext/MLIRCUDAExt.jl:154-161): tuples, default
    workgroup ``min(256, ndrange[1])`` along dim 1."""
    if isinstance(ndrange, (int, np.integer)):
        ndrange = (int(ndrange),)
    if isinstance(workgroupsize, (int, np.integer)):
        workgroupsize = (int(workgroupsize),)
    ndrange = tuple(ndrange)
    if workgroupsize is None:
        workgroupsize = tuple(min(256, ndrange[0]) if d == 0 else 1 for d in range(len(ndrange)))
    return ndrange, tuple(workgroupsize), None, None


def as_tuple(x: int | Iterable[int]) -> tuple[int, ...]:
    if isinstance(x, (int, np.integer)):
        return (int(x),)
    return tuple(int(v) for v in x)
