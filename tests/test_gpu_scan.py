"""Prefix scan (mk_accumulate_f32) against the fp64 oracle: AK.accumulate! and
cumsum (test/test_downstream_ka.jl:39-42 inclusive of 1:n, :75-78 exclusive).
Bar: each output within 1e-6 of the running sum of |x| (one Float32 rounding
of an fp64 carry); max/min exact."""
import operator
import os
import sys

import numpy as np
import pytest
import torch

import cutilecpu_b200 as mk
import oracle
from cutilecpu_b200 import _lib

pytestmark = pytest.mark.gpu


def scan(x: np.ndarray, op="add", init=0.0, exclusive=False, off=0, inplace=False) -> np.ndarray:
    xd = torch.from_numpy(np.concatenate([np.zeros(off, np.float32), x])).cuda()
    out = xd if inplace else torch.full_like(xd, np.nan)
    rc = _lib.lib().mk_accumulate_f32(out.data_ptr() + 4 * off, xd.data_ptr() + 4 * off, x.size, _lib.MK_OP[op],
                                      float(init), int(exclusive), torch.cuda.current_stream().cuda_stream)
    assert rc == 0, _lib.last_error()
    assert _lib.lib().mk_error_poll(torch.cuda.current_stream().cuda_stream) == 0
    return out.cpu().numpy()[off:]


def check_add(got, x, init=0.0, exclusive=False):
    want = oracle.accumulate(x, "add", init, exclusive)
    scale = np.abs(init) + np.cumsum(np.abs(x.astype(np.float64)))
    assert np.all(np.abs(got - want) <= 1e-6 * scale + 1e-30)


def test_cumsum_1_to_1024(cuda):
    x = np.arange(1, 1025, dtype=np.float32)
    np.testing.assert_array_equal(scan(x), np.cumsum(np.arange(1, 1025)).astype(np.float32))


# 8192: one 256-row tile; 8197: a second tile holding only the partial row;
# 3*8192 + 233: ragged last tile with a partial row
@pytest.mark.parametrize("n", [1, 2, 31, 4095, 4096, 4097, 8192, 8197, 3 * 8192 + 233, 100_000, (1 << 22) + 7,
                               1 << 26])
@pytest.mark.parametrize("exclusive", [False, True])
def test_scan_add_sizes(cuda, n, exclusive):
    r = np.random.Generator(np.random.Philox(n))
    x = (r.random(n, dtype=np.float32) * 2 - 1).astype(np.float32)
    check_add(scan(x, exclusive=exclusive, init=0.5), x, 0.5, exclusive)


@pytest.mark.parametrize("op,init", [("max", -np.inf), ("min", np.inf)])
def test_scan_max_min_exact(cuda, op, init):
    r = np.random.Generator(np.random.Philox(7))
    x = r.standard_normal(300_001, dtype=np.float32)
    np.testing.assert_array_equal(scan(x, op, init), oracle.accumulate(x, op, init).astype(np.float32))


@pytest.mark.parametrize("n", [8197, 300_001])
def test_scan_mul_exact(cuda, n):
    r = np.random.Generator(np.random.Philox(10))
    x = np.where(r.random(n) < 0.5, -1.0, 1.0).astype(np.float32)  # products stay exactly +-1
    for exclusive in (False, True):
        np.testing.assert_array_equal(scan(x, "mul", 1.0, exclusive),
                                      oracle.accumulate(x, "mul", 1.0, exclusive).astype(np.float32))


def test_scan_inplace_exclusive_ragged(cuda):
    r = np.random.Generator(np.random.Philox(11))
    x = r.random((1 << 20) + 29, dtype=np.float32)
    check_add(scan(x, inplace=True, exclusive=True, init=2.0), x, 2.0, True)


def test_scan_misaligned_and_inplace(cuda):
    r = np.random.Generator(np.random.Philox(8))
    x = r.random(50_001, dtype=np.float32)
    check_add(scan(x, off=3), x)
    check_add(scan(x, inplace=True), x)


def test_scan_deterministic_property_full_size(cuda):
    # size-independent property: the last inclusive value equals the sum
    r = np.random.Generator(np.random.Philox(9))
    n = 1 << 28
    x = r.random(n, dtype=np.float32)
    got = scan(x)
    assert abs(float(got[-1]) - oracle.mapreduce(x)) <= 1e-6 * oracle.mapreduce(x)
    assert np.all(np.diff(got[::4096]) >= 0)  # non-negative inputs: non-decreasing


def test_surface_accumulate_and_cumsum(cuda):
    src = mk.MLIRArray(np.arange(1, 1025, dtype=np.float32))
    dst = mk.zeros(mk.get_backend(src), "Float32", 1024)
    mk.accumulate(operator.add, dst, src, init=0.0)
    np.testing.assert_array_equal(mk.Array(dst), np.cumsum(np.arange(1, 1025)).astype(np.float32))
    np.testing.assert_array_equal(mk.Array(mk.cumsum(src)), mk.Array(dst))
    ex = mk.zeros(mk.get_backend(src), "Float32", 1024)
    mk.accumulate(operator.add, ex, src, init=0.0, inclusive=False)
    np.testing.assert_array_equal(mk.Array(ex)[1:], mk.Array(dst)[:-1])


_TIMEOUT_CHILD = r"""
import sys
import numpy as np, torch
sys.path.insert(0, sys.argv[1])
from cutilecpu_b200 import _lib
L = _lib.lib()
n = 1 << 26
x = torch.rand(n, device="cuda")
y = torch.empty_like(x)
s = torch.cuda.current_stream().cuda_stream
assert L.mk_accumulate_f32(y.data_ptr(), x.data_ptr(), n, 0, 0.0, 0, s) == 0, _lib.last_error()
rc = L.mk_error_poll(s)
print("POLL", rc, _lib.last_error())
# the context stays usable after the timeout: a plain kernel still runs
z = torch.ones(1024, device="cuda").sum().item()
print("AFTER", z)
"""


def test_lookback_wait_runs_out_and_reports_timeout(cuda, tmp_path):
    """The look-back wait is bounded: with a budget of one SM cycle
    (MK_WAIT_LIMIT_CYCLES=1) the tiles that find a predecessor unpublished give
    up, publish a prefix anyway (so no successor waits forever) and raise the
    timeout bit, which mk_error_poll reports as MK_ERR_TIMEOUT, the library's
    counterpart of the KernelException the reference raises for a device
    error (test/test_gpu_simt.jl:497-565).  Runs in a child process because
    the limit is read once per process; a fresh child then scans normally."""
    import subprocess
    from conftest import ROOT
    script = tmp_path / "child.py"
    script.write_text(_TIMEOUT_CHILD)
    env = dict(os.environ, MK_WAIT_LIMIT_CYCLES="1")
    r = subprocess.run([sys.executable, str(script), str(ROOT)], env=env, capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    poll = [ln for ln in r.stdout.splitlines() if ln.startswith("POLL")][0].split()
    assert int(poll[1]) == _lib.MK_ERR_TIMEOUT, r.stdout
    assert "timed out" in r.stdout
    assert "AFTER 1024.0" in r.stdout
    # and without the tiny limit (this process, default budget) the same size is right
    x = np.random.Generator(np.random.Philox(5)).random(1 << 26, dtype=np.float32)
    check_add(scan(x), x)
