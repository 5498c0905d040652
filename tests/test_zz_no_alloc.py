"""The allocation-free FFT entry point, checked against the planned FFT.

cubutterflyB200FftC2CNoAlloc serves callers that cannot allocate device
memory (fixed budgets, pools that own every byte, hosts that forbid
cudaMalloc on their threads) and therefore cannot hand a planned multi-pass
FFT its workspace: it keeps its scratch in a device array inside the library.
Here it is called through the C ABI twice in a row and each result is compared
with cubutterflyCreatePlan/Execute (caller workspace) at the FFT tolerance.
The file sorts last so a stop-at-first-failure run has run everything else
first; it also passes on its own in a fresh process.
"""
import ctypes as ct

import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
TOL = 2e-6  # relative L2, fp32 FFT


def bind(lib):
    fn = lib._dll.cubutterflyB200FftC2CNoAlloc
    fn.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_size_t, ct.c_int, ct.c_int, ct.c_void_p]
    fn.restype = ct.c_int
    return fn


def planned(lib, x, inverse, in_place, cuda):
    from gpu_util import run

    t = cb.Transform(op=cb.Operator.FFT, extents=[x.shape[1]], batch=x.shape[0], inverse=inverse,
                     normalize_inverse=True, in_place=in_place)
    got, name = run(lib, t, x, cuda)
    assert name.startswith("fft-stockham-global")
    return got


def no_alloc(lib, fn, x, inverse, in_place, cuda):
    stream = torch.cuda.current_stream().cuda_stream
    din = torch.from_numpy(x.view(np.float32).copy()).to(cuda)
    dout = din if in_place else torch.empty_like(din)
    status = fn(din.data_ptr(), dout.data_ptr(), x.shape[1], x.shape[0], int(inverse), 1, stream)
    assert status == 0, lib._dll.cubutterflyGetLastErrorString()
    torch.cuda.synchronize()
    return dout.cpu().numpy().view(np.complex64).reshape(x.shape)


def test_no_alloc_matches_planned_two_calls(lib, cuda):
    fn = bind(lib)
    # call 1: 2^16 x 4 in place, forward (two passes); call 2: 2^21 x 1 out of
    # place, inverse with 1/N (three passes), reusing the scratch of call 1
    cases = [(16, 4, False, True), (21, 1, True, False)]
    for log_n, batch, inverse, in_place in cases:
        x = w.fft_input(1 << log_n, batch, seed=log_n)
        want = planned(lib, x, inverse, in_place, cuda)
        got = no_alloc(lib, fn, x, inverse, in_place, cuda)
        assert rel_l2(got, want) <= TOL


def test_no_alloc_rejects_sizes_beyond_its_scratch(lib, cuda):
    fn = bind(lib)
    buf = torch.empty(2, dtype=torch.float32, device=cuda)
    too_long = fn(buf.data_ptr(), buf.data_ptr(), 1 << 22, 1, 0, 1, 0)
    assert too_long == cb.Status.INVALID_VALUE
    assert b"2^14 .. 2^21" in lib._dll.cubutterflyGetLastErrorString()
    too_many = fn(buf.data_ptr(), buf.data_ptr(), 1 << 16, 64, 0, 1, 0)
    assert too_many == cb.Status.INVALID_VALUE
    assert b"16 MiB" in lib._dll.cubutterflyGetLastErrorString()
