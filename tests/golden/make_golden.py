"""Generate the golden known-answer fixtures of tests/golden/*.npz.

The reference ships no golden-vector files; its tests compute expected values
inline from closed forms or from Base Julia on the same host inputs.  Each
fixture below restates one of those known-answer tests, with the expected
output computed independently of the C oracle (numpy fp32/fp64 arithmetic or a
closed form), so the oracle is pinned against it:

  vadd_4096          test/test_gpu_simt.jl:322-328   c == a .+ b (exact)
  vadd_tail_1000     test/test_gpu_simt.jl:441-446   masked tail, exact
  vadd_tail_257      test/test_gpu_simt.jl:441-446   masked tail, exact
  hist_ka_4096_256   test/test_gpu_simt.jl:353-359   KA histogram, exact
  hist_mod_4096_8    test/test_ka_cpu.jl:67-72       all bins == N ÷ NB
  hist_one_65536     test/test_ka_cpu.jl:75-79       one slot == 65536
  reduce_1_1024      test/test_downstream_ka.jl:27-31 sum(1:1024) == 524800
  gpuarrays_1024     test/test_gpuarrays.jl:51,83-91  sum/max/min/sum(abs2)/prod/count(>(0))
  mm_tiled_256       test/test_gpu_simt.jl:407-413   C ≈ A*B (fp64 expected)
  gather_perm_4096   gather KAT: a = 1:n, c[i] == idx[i] (closed form)

Run from the repository root:  python tests/golden/make_golden.py
"""
from __future__ import annotations

from pathlib import Path

import numpy as np

OUT = Path(__file__).resolve().parent


def g(seed: int) -> np.random.Generator:
    return np.random.Generator(np.random.Philox(key=seed))


def main() -> None:
    r = g(1)
    a = r.random(4096, dtype=np.float32)
    b = r.random(4096, dtype=np.float32)
    np.savez_compressed(OUT / "vadd_4096.npz", a=a, b=b, c=(a + b).astype(np.float32))
    for n in (1000, 257):
        a = r.random(n, dtype=np.float32)
        b = r.random(n, dtype=np.float32)
        np.savez_compressed(OUT / f"vadd_tail_{n}.npz", a=a, b=b, c=(a + b).astype(np.float32))

    keys = r.integers(1, 257, size=4096, dtype=np.int32)
    np.savez_compressed(OUT / "hist_ka_4096_256.npz", keys=keys, nbins=np.int32(256),
             counts=np.bincount(keys - 1, minlength=256).astype(np.uint32))
    keys = np.array([(j % 8) + 1 for j in range(4096)], dtype=np.int32)
    np.savez_compressed(OUT / "hist_mod_4096_8.npz", keys=keys, nbins=np.int32(8),
             counts=np.full(8, 4096 // 8, dtype=np.uint32))
    np.savez_compressed(OUT / "hist_one_65536.npz", keys=np.ones(65536, dtype=np.int32), nbins=np.int32(1),
             counts=np.array([65536], dtype=np.uint32))

    x = np.arange(1, 1025, dtype=np.float32)
    np.savez_compressed(OUT / "reduce_1_1024.npz", x=x, sum=np.float64(1024 * 1025 // 2))

    a = r.random(1024, dtype=np.float32)
    p = (r.random(1024, dtype=np.float32) + np.float32(0.5)).astype(np.float32)
    a64, p64 = a.astype(np.float64), p.astype(np.float64)
    s = (a - np.float32(0.5)).astype(np.float32)  # count(>(0.5), a) == count(>(0), a .- 0.5f0)
    np.savez_compressed(OUT / "gpuarrays_1024.npz", a=a, p=p,
             sum=a64.sum(), maximum=np.float64(a.max()), minimum=np.float64(a.min()),
             sum_abs2=(a64 * a64).sum(), prod=np.prod(p64),
             s=s, count_s_gt0=np.int64((s > 0).sum()))

    n = 256
    A = np.asfortranarray(r.random((n, n), dtype=np.float32))
    B = np.asfortranarray(r.random((n, n), dtype=np.float32))
    np.savez_compressed(OUT / "mm_tiled_256.npz", A=A, B=B, C=A.astype(np.float64) @ B.astype(np.float64))

    n = 4096
    idx = (r.permutation(n) + 1).astype(np.int32)
    np.savez_compressed(OUT / "gather_perm_4096.npz", a=np.arange(1, n + 1, dtype=np.float32), idx=idx,
             c=idx.astype(np.float32))


if __name__ == "__main__":
    main()
