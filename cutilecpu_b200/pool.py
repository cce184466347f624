"""Memory pools of libkernels.so, exposed as MLIRArrays and host arrays.

* ``pool_allocate(T, dims)``: an MLIRArray over device memory from the
  library's per-device stream-ordered pool (the counterpart of CUDA.jl's pool
  behind ``KA.allocate``, ext/MLIRCUDAExt.jl:140).  The tensor is a zero-copy
  view (``__cuda_array_interface__``); the block returns to the pool when the
  array is garbage collected.
* ``aligned_array(T, dims, alignment=64)``: a host numpy array in pinned,
  page-aligned memory with the argument checks of the reference's
  ``aligned_array`` (src/allocator.jl:32-61); pinned buffers make H2D/D2H
  copies asynchronous and full-speed.
"""
from __future__ import annotations

import ctypes as C
import math
import weakref

import numpy as np
import torch

from . import _lib
from .array import ELTYPES, MLIRArray, _dims, current_stream_handle, eltype_name


class _DeviceBlock:
    """Owner of one pool block; exposes it through ``__cuda_array_interface__``."""

    def __init__(self, ptr: int, nbytes: int, typestr: str, shape: tuple[int, ...], stream: int):
        self.ptr, self.nbytes, self.stream = ptr, nbytes, stream
        self.__cuda_array_interface__ = {"shape": shape, "typestr": typestr, "data": (ptr, False),
                                         "version": 3, "strides": None}


def _free_device(ptr: int, stream: int) -> None:
    try:
        _lib.lib().mk_pool_free_device(ptr, stream)
    except Exception:  # interpreter shutdown
        pass


def pool_allocate(T, dims) -> MLIRArray:
    """An uninitialised MLIRArray in pool memory on the current device."""
    name = eltype_name(T)
    d = _dims(dims)
    n = math.prod(d)
    npdt, tdt = ELTYPES[name]
    nbytes = max(1, n) * npdt.itemsize
    p = C.c_void_p()
    stream = current_stream_handle()
    _lib.check(_lib.lib().mk_pool_alloc_device(C.byref(p), nbytes, stream), "pool_allocate")
    typestr = np.dtype(np.int32 if name == "UInt32" else npdt).str
    block = _DeviceBlock(p.value, nbytes, typestr, (n,), stream)
    t = torch.as_tensor(block, device="cuda")
    assert t.data_ptr() == p.value, "pool_allocate: torch copied the block"
    weakref.finalize(t, _free_device, p.value, stream)
    return MLIRArray(t, dims=d, eltype=name)


def _check_alignment(alignment: int) -> None:
    """The checks of src/allocator.jl:52-61 (done here so they raise without a GPU)."""
    if alignment <= 0:
        raise ValueError(f"alignment must be positive, got {alignment}")
    if alignment & (alignment - 1):
        raise ValueError(f"alignment must be a power of two, got {alignment}")
    if alignment % C.sizeof(C.c_void_p):
        raise ValueError(f"alignment ({alignment}) must be a multiple of sizeof(Ptr{{Cvoid}}) "
                         f"(={C.sizeof(C.c_void_p)})")


def _free_host(ptr: int) -> None:
    try:
        _lib.lib().mk_host_free(ptr)
    except Exception:
        pass


def aligned_array(T, dims, alignment: int = 64) -> np.ndarray:
    """A pinned host array whose data pointer is ``alignment``-aligned."""
    _check_alignment(alignment)
    npdt = ELTYPES[eltype_name(T)][0]
    d = _dims(dims)
    nbytes = max(1, math.prod(d)) * npdt.itemsize
    p = C.c_void_p()
    _lib.check(_lib.lib().mk_host_alloc_aligned(C.byref(p), nbytes, alignment), "aligned_array")
    buf = (C.c_char * nbytes).from_address(p.value)
    arr = np.frombuffer(buf, dtype=npdt, count=math.prod(d)).reshape(d, order="F")
    weakref.finalize(buf, _free_host, p.value)
    return arr


def pointer_aligned(a: np.ndarray, alignment: int) -> bool:
    """``pointer_aligned(a, alignment)`` (src/allocator.jl:70-71)."""
    return a.ctypes.data % alignment == 0


def pool_stats() -> dict:
    vals = [C.c_size_t() for _ in range(4)]
    _lib.check(_lib.lib().mk_pool_stats(*[C.byref(v) for v in vals]), "pool_stats")
    keys = ("device_reserved", "device_used", "pinned_live", "pinned_cached")
    return {k: v.value for k, v in zip(keys, vals)}


def pool_trim() -> None:
    _lib.check(_lib.lib().mk_pool_trim(), "pool_trim")
