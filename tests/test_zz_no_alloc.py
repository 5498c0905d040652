"""The allocation-free FFT entry point, checked against the planned FFT and the oracle.

cubutterflyB200FftC2CNoAlloc serves callers that cannot allocate device
memory (fixed budgets, pools that own every byte, hosts that forbid
cudaMalloc on their threads) and therefore cannot hand a planned multi-pass
FFT its workspace: it keeps its scratch in a device array inside the library.
Each case calls it through the C ABI twice in a row and compares both results
with cubutterflyCreatePlan/Execute (caller workspace) at the FFT tolerance;
the two ends of its length range are also held to the CPU oracle directly.
The file sorts last so a stop-at-first-failure run has run everything else
first; it also passes on its own in a fresh process.
"""
import ctypes as ct
import os
import subprocess
import sys
import textwrap
from pathlib import Path

import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
TOL = 2e-6  # relative L2, fp32 FFT
ROOT = Path(__file__).resolve().parents[1]


def bind(lib):
    fn = lib._dll.cubutterflyB200FftC2CNoAlloc
    fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_size_t, ct.c_int, ct.c_int, ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def planned(lib, x, inverse, normalize, in_place, cuda):
    from gpu_util import run

    t = cb.Transform(op=cb.Operator.FFT, extents=[x.shape[1]], batch=x.shape[0], inverse=inverse,
                     normalize_inverse=normalize, in_place=in_place)
    got, name = run(lib, t, x, cuda)
    assert name.startswith("fft-stockham-global")
    return got


def no_alloc(lib, fn, x, inverse, normalize, in_place, cuda):
    stream = torch.cuda.current_stream().cuda_stream
    din = torch.from_numpy(x.view(np.float32).copy()).to(cuda)
    dout = din if in_place else torch.empty_like(din)
    status = fn(din.data_ptr(), dout.data_ptr(), x.shape[1], x.shape[0], int(inverse), int(normalize), stream)
    assert status == 0, lib._dll.cubutterflyGetLastErrorString()
    torch.cuda.synchronize()
    return dout.cpu().numpy().view(np.complex64).reshape(x.shape)


# (log n, batch, inverse, normalize, in place): both pass counts (two passes up
# to 2^20, three at 2^21), the shortest length (7 + 7-bit passes), inverse with
# and without 1/N, in place, and batches at the scratch limit (n * batch = 2^21)
CASES = [
    (14, 2, False, True, False),
    (14, 128, True, False, True),
    (16, 4, False, True, True),
    (17, 16, False, True, False),
    (17, 16, True, True, True),
    (20, 2, True, True, True),
    (21, 1, True, True, False),
    (21, 1, False, True, False),
]


@pytest.mark.parametrize("log_n,batch,inverse,normalize,in_place", CASES)
def test_no_alloc_matches_planned_two_calls(lib, cuda, log_n, batch, inverse, normalize, in_place):
    fn = bind(lib)
    x = w.fft_input(1 << log_n, batch, seed=log_n + batch)
    want = planned(lib, x, inverse, normalize, in_place, cuda)
    for _ in range(2):  # the second call reuses the scratch the first one left behind
        got = no_alloc(lib, fn, x, inverse, normalize, in_place, cuda)
        assert rel_l2(got, want) <= TOL


@pytest.mark.parametrize("log_n,inverse", [(14, False), (21, True)])
def test_no_alloc_range_ends_match_the_oracle(lib, cuda, oracle, log_n, inverse):
    fn = bind(lib)
    x = w.fft_input(1 << log_n, 1, seed=100 + log_n)
    got = no_alloc(lib, fn, x, inverse, True, False, cuda)
    assert rel_l2(got, oracle.fft_c32(x, inverse=inverse, normalize=True)) <= TOL


def test_no_alloc_rejects_sizes_beyond_its_scratch(lib, cuda):
    fn = bind(lib)
    buf = torch.empty(1 << 22, dtype=torch.float32, device=cuda)
    too_long = fn(buf.data_ptr(), buf.data_ptr(), 1 << 22, 1, 0, 1, 0)
    assert too_long == cb.Status.INVALID_VALUE
    assert b"2^14 .. 2^21" in lib._dll.cubutterflyGetLastErrorString()
    too_many = fn(buf.data_ptr(), buf.data_ptr(), 1 << 16, 64, 0, 1, 0)
    assert too_many == cb.Status.INVALID_VALUE
    assert b"16 MiB" in lib._dll.cubutterflyGetLastErrorString()
    # in place, 2^21 points take three passes and would need 32 MiB of scratch
    in_place_max = fn(buf.data_ptr(), buf.data_ptr(), 1 << 21, 1, 0, 1, 0)
    assert in_place_max == cb.Status.INVALID_VALUE
    assert b"out of place" in lib._dll.cubutterflyGetLastErrorString()


def test_no_alloc_rejects_partly_overlapping_buffers(lib, cuda):
    fn = bind(lib)
    buf = torch.empty(2 * (1 << 15), dtype=torch.float32, device=cuda)  # 2^15 complex values
    status = fn(buf.data_ptr(), buf.data_ptr() + 8 * 1024, 1 << 14, 1, 0, 1, 0)
    assert status == cb.Status.INVALID_VALUE
    assert b"overlap" in lib._dll.cubutterflyGetLastErrorString()


FIRST_CALL_SCRIPT = textwrap.dedent("""
    import ctypes as ct, sys
    import numpy as np, torch
    sys.path.insert(0, sys.argv[1]); sys.path.insert(0, sys.argv[1] + "/tests")
    import cubutterfly_b200 as cb
    from cubutterfly_b200 import workloads as w
    from conftest import rel_l2
    from oracle.oracle import Oracle
    lib = cb.Library()
    fn = lib._dll.cubutterflyB200FftC2CNoAlloc
    fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_size_t, ct.c_int, ct.c_int, ct.c_void_p]
    fn.restype = ct.c_int
    side = torch.cuda.Stream()  # torch pool streams are non-blocking
    x = w.fft_input(1 << 15, 2, seed=9)
    with torch.cuda.stream(side):
        din = torch.from_numpy(x.view(np.float32).copy()).to("cuda", non_blocking=False)
        dout = torch.empty_like(din)
        status = fn(din.data_ptr(), dout.data_ptr(), 1 << 15, 2, 0, 1, side.cuda_stream)
        assert status == 0, lib._dll.cubutterflyGetLastErrorString()
    side.synchronize()
    got = dout.cpu().numpy().view(np.complex64).reshape(x.shape)
    err = rel_l2(got, Oracle().fft_c32(x))
    assert err <= 2e-6, err
    print("first call ok", err)
""")


def test_no_alloc_first_call_on_a_non_blocking_stream(cuda):
    """The one-time table upload must be complete before the first call's
    kernels run, even when they run on a stream that does not wait for the
    legacy default stream: a fresh process makes its first call there."""
    env = dict(os.environ)
    r = subprocess.run([sys.executable, "-c", FIRST_CALL_SCRIPT, str(ROOT)], capture_output=True, text=True,
                       timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "first call ok" in r.stdout
