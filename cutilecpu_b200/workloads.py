"""Seeded synthetic inputs for the five benchmark configurations.

The reference publishes no datasets for this path; its benchmark inputs are
``rand``/``randn`` arrays (examples/tiled_matmul.jl:61-64,
examples/reflection_and_perf.jl:66-77).  The configurations are:

=========  ==========================================================  ==========
name       input                                                        size
=========  ==========================================================  ==========
vadd       a, b ~ U[0,1) Float32                                        n = 2^20
reduce     x ~ U[-1,1) Float32, sum(x.^2)                               n = 2^28
gather     a ~ U[0,1) Float32 (2^27), idx ~ U{1..2^27} Int32 (2^27)     n = 2^27
histogram  keys ~ Zipf(s=1.1) on 1..4096 Int32, UInt32 counts           n = 2^26
matmul     A, B ~ N(0,1) Float32, C = A*B                               8192^3
=========  ==========================================================  ==========

All inputs come from numpy's counter-based Philox generator with a fixed
seed, on the host, so every consumer (GPU kernels, CPU oracle, CPU baseline)
sees identical bits.
"""
from __future__ import annotations

import numpy as np

SEED = 20240601

CONFIGS = {
    "vadd": {"n": 1 << 20, "wg": 256},
    "reduce": {"n": 1 << 28},
    "gather": {"n": 1 << 27, "na": 1 << 27},
    "histogram": {"n": 1 << 26, "nbins": 4096, "s": 1.1},
    "matmul": {"m": 8192, "n": 8192, "k": 8192},
}


def rng(seed: int = SEED, stream: int = 0) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=seed + 7919 * stream))


def uniform01(n: int, seed: int = SEED, stream: int = 0) -> np.ndarray:
    return rng(seed, stream).random(n, dtype=np.float32)


def uniform_pm1(n: int, seed: int = SEED, stream: int = 1) -> np.ndarray:
    u = rng(seed, stream).random(n, dtype=np.float32)
    u *= 2.0
    u -= 1.0
    return u


def indices1(n: int, na: int, seed: int = SEED, stream: int = 2) -> np.ndarray:
    """1-based Int32 indices uniform in [1, na]."""
    return rng(seed, stream).integers(1, na + 1, size=n, dtype=np.int32)


def zipf_keys(n: int, nbins: int = 4096, s: float = 1.1, seed: int = SEED, stream: int = 3) -> np.ndarray:
    """1-based Int32 keys with P(k) proportional to k^-s on 1..nbins (inverse CDF)."""
    w = np.arange(1, nbins + 1, dtype=np.float64) ** (-s)
    cdf = np.cumsum(w)
    cdf /= cdf[-1]
    u = rng(seed, stream).random(n)
    k = np.searchsorted(cdf, u, side="right")
    np.minimum(k, nbins - 1, out=k)
    return (k + 1).astype(np.int32)


def normal(shape, seed: int = SEED, stream: int = 4) -> np.ndarray:
    """Standard normal Float32 in Fortran (column-major) order."""
    g = rng(seed, stream)
    x = g.standard_normal(int(np.prod(shape)), dtype=np.float32)
    return x.reshape(shape, order="F")
