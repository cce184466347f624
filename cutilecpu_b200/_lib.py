"""ctypes binding of ``libkernels.so`` (the C ABI declared in include/mk_kernels.h).

The library is built in-tree (``python -m cutilecpu_b200.csrc.build``).  There
is no fallback: if the shared object is missing or does not load, every call
raises, so a GPU run can never silently take another path.
"""
from __future__ import annotations

import ctypes as C
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libkernels.so"

MK_OK = 0
MK_ERR_INVALID = -1
MK_ERR_CUDA = -2
MK_ERR_NCCL = -3
MK_ERR_TIMEOUT = -4
MK_ERR_DEVICE_FAULT = -5

MK_F = {"identity": 0, "abs2": 1, "abs": 2, "gt0": 3}
MK_OP = {"add": 0, "max": 1, "min": 2, "mul": 3}

# name -> (restype, argtypes); keep in step with include/mk_kernels.h
_i64, _i32, _f64, _vp, _int = C.c_int64, C.c_int32, C.c_double, C.c_void_p, C.c_int
SIGNATURES = {
    "mk_version": (_int, []),
    "mk_last_error": (C.c_char_p, []),
    "mk_init": (_int, [_int]),
    "mk_error_poll": (_int, [_vp]),
    "mk_vadd_f32": (_int, [_vp, _vp, _vp, _i64, _vp]),
    "mk_probe_vadd_f32": (_int, [_int, _vp, _vp, _vp, _i64, _vp, _vp]),
    "mk_axpby_f32": (_int, [_vp, C.c_float, _vp, C.c_float, _vp, _i64, _vp]),
    "mk_mapreduce_f32": (_int, [_vp, _vp, _i64, _int, _int, _f64, _vp]),
    "mk_sum_sq_f32": (_int, [_vp, _vp, _i64, _vp]),
    "mk_mapreduce_f32_noalloc": (_int, [_vp, _vp, _i64, _int, _int, _f64, _vp]),
    "mk_mapreduce_dim_f32": (_int, [_vp, _vp, _i64, _i64, _i64, _int, _int, _f64, _vp]),
    "mk_accumulate_f32": (_int, [_vp, _vp, _i64, _int, _f64, _int, _vp]),
    "mk_findext_f32": (_int, [_vp, _vp, _vp, _i64, _int, _vp]),
    "mk_gather_f32": (_int, [_vp, _vp, _i64, _vp, _i64, _vp]),
    "mk_probe_random_read_f32": (_int, [_vp, _i64, _vp, _i64, _i64, C.c_uint, _vp]),
    "mk_hist_u32": (_int, [_vp, _i32, _vp, _i64, _vp]),
    "mk_hist": (_int, [_vp, _int, _i32, _vp, _int, _i64, _vp]),
    "mk_sgemm_3xtf32": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mk_sgemm_f32": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mk_matmul_tiled16_f32": (_int, [_vp, _vp, _vp, _i64, _i64, _i64, _i64, _i64, _i64, _vp]),
    "mk_peer_handle_size": (_int, []),
    "mk_peer_create": (_int, [_int, _int, _vp]),
    "mk_peer_connect": (_int, [_vp]),
    "mk_peer_destroy": (_int, []),
    "mk_mapreduce_f32_allreduce": (_int, [_vp, _vp, _i64, _int, _int, _f64, _vp]),
    "mk_mapreduce_f32_allreduce_async": (_int, [_vp, _vp, _i64, _int, _int, _f64, _vp]),
    "mk_allreduce_complete": (_int, [_vp]),
    "mk_peer_trace": (_int, [_vp, _int]),
    "mk_hist_u32_allreduce": (_int, [_vp, _vp, _i32, _vp, _i64, _vp]),
    "mk_hist_u32_allreduce_async": (_int, [_vp, _vp, _i32, _vp, _i64, _vp]),
    "mk_hist_allreduce_complete": (_int, [_vp]),
    "mk_pool_alloc_device": (_int, [C.POINTER(C.c_void_p), C.c_size_t, _vp]),
    "mk_pool_free_device": (_int, [_vp, _vp]),
    "mk_host_alloc_aligned": (_int, [C.POINTER(C.c_void_p), C.c_size_t, C.c_size_t]),
    "mk_host_free": (_int, [_vp]),
    "mk_pool_stats": (_int, [C.POINTER(C.c_size_t)] * 4),
    "mk_pool_trim": (_int, []),
}


class MLIRKernelsError(RuntimeError):
    """A launch was rejected (bad argument) or a CUDA call failed."""


class KernelException(MLIRKernelsError):
    """A kernel flagged bad input on the device (out-of-range index / key).

    Mirrors the KernelException that CUDA.jl raises at the next synchronize
    when a reference kernel throws (src/lower.jl:1673-1703).
    """


_lib: C.CDLL | None = None


def lib() -> C.CDLL:
    """Load libkernels.so once; raise if it is absent (no fallback path)."""
    global _lib
    if _lib is None:
        if not LIB_PATH.exists():
            raise MLIRKernelsError(
                f"{LIB_PATH} is not built; run `python -m cutilecpu_b200.csrc.build`")
        L = C.CDLL(str(LIB_PATH))
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = res
            fn.argtypes = args
        _lib = L
    return _lib


def last_error() -> str:
    msg = lib().mk_last_error()
    return msg.decode() if msg else ""


def check(rc: int, what: str) -> None:
    """Raise the Python counterpart of a non-zero status."""
    if rc == MK_OK:
        return
    msg = last_error() or f"status {rc}"
    if rc in (MK_ERR_DEVICE_FAULT, MK_ERR_TIMEOUT):
        raise KernelException(f"{what}: {msg}")
    raise MLIRKernelsError(f"{what}: {msg}")
