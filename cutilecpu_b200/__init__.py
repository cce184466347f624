"""cutilecpu_b200 — B200 (sm_100a) kernels for the MLIRKernels.jl hot path.

The Python side mirrors the KernelAbstractions surface the reference exposes
(``MLIRCUDABackend``, ``MLIRArray``, ``get_backend``, ``allocate``, kernel
launches with ``ndrange``/``workgroupsize``, AK/GPUArrays reductions); every
computation runs in ``libkernels.so`` (C ABI: include/mk_kernels.h).
"""
from ._lib import KernelException, MLIRKernelsError
from .array import (Array, MLIRArray, MLIRCUDABackend, allocate, copyto, functional, get_backend,
                    launch_config, ones, supports_atomics, synchronize, zeros)
from .kernels import Kernel, KernelFunction, Scale, axpby, gather, map_, histogram, mm_naive, mm_tiled, mm_tiled_simt, mul, vadd
from .reductions import (Broadcasted, abs2, accumulate, all_, any_, argmax, argmin, cumsum, extrema, findmax,
                         findmin, count, identity, mapreduce, mapreducedim, maximum, minimum,
                     positive, prod, reduce, sum)
from . import distributed, reductions
from .pool import aligned_array, pointer_aligned, pool_allocate, pool_stats, pool_trim

__all__ = [
    "KernelException", "MLIRKernelsError", "Array", "MLIRArray", "MLIRCUDABackend", "allocate",
    "copyto", "functional", "get_backend", "launch_config", "ones", "supports_atomics", "synchronize",
    "zeros", "Kernel", "KernelFunction", "Scale", "axpby", "map_", "gather", "histogram", "mm_naive", "mm_tiled", "mm_tiled_simt", "mul", "vadd", "Broadcasted",
    "abs2", "accumulate", "all_", "any_", "argmax", "argmin", "cumsum", "extrema", "findmax", "findmin", "count", "identity", "mapreduce", "mapreducedim", "maximum", "minimum", "positive", "prod",
    "reduce", "sum", "distributed", "aligned_array", "pointer_aligned", "pool_allocate", "pool_stats",
    "pool_trim",
]
