"""Back-to-back executions whose inputs are the previous execution's outputs.

The column-pair and global FFT passes, the FWHT and bitwise tiles and the
zeta chain steps launch as programmatic dependents of the kernel before them
on the stream: their CTAs may be scheduled while that kernel finishes and wait
for it (griddepcontrol.wait) before touching memory.  These tests enqueue long
dependent sequences -- forward and inverse transforms feeding each other,
with an ordinary torch kernel in between -- with no synchronisation, and check
the end results against the CPU oracle: a kernel that read its input before the
producer had finished would fail them.
"""
import numpy as np
import pytest

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu

TOL = 2e-6  # relative L2, fp32 FFT


def _fft(n, batch, inverse=False):
    return cb.Transform(op=cb.Operator.FFT, extents=[n], batch=batch, inverse=inverse, normalize_inverse=True)


def _rel_dev(a, b):
    import torch

    a, b = a.double(), b.double()
    return float(torch.linalg.vector_norm(a - b) / torch.linalg.vector_norm(b))


@pytest.mark.parametrize("log_n, batch", [(12, 1024), (26, 1)])
def test_fft_dependent_chain(lib, oracle, cuda, log_n, batch):
    """Config-0 shape (one column-pair launch per call) and a 2^26-point
    transform (four global passes per call): F, F^-1, F, ... ten calls, each
    reading the previous call's output, every other step scaled by 1 by a
    torch kernel; the last forward output against the oracle's FFT of x and
    the final inverse output against x (rel L2 <= 2e-6)."""
    import torch

    n = 1 << log_n
    x = w.torch_fft_input(n, batch, cuda, seed=31).reshape(n * batch, 2)
    stream = torch.cuda.current_stream().cuda_stream
    with cb.Plan(lib, _fft(n, batch), stream=stream) as fwd, \
            cb.Plan(lib, _fft(n, batch, inverse=True), stream=stream) as inv:
        wss = []
        for p in (fwd, inv):
            if p.workspace_size():
                wss.append(torch.empty(p.workspace_size(), dtype=torch.uint8, device=cuda))
                p.set_workspace(wss[-1].data_ptr(), p.workspace_size())
        a, b = torch.empty_like(x), torch.empty_like(x)
        src = x
        for i in range(10):
            dst = a if i % 2 == 0 else b
            (fwd if i % 2 == 0 else inv).execute(src.data_ptr(), dst.data_ptr())
            if i % 4 == 1:
                dst.mul_(1.0)
            src = dst
        last_fwd = a.clone()
        torch.cuda.synchronize()
    assert _rel_dev(b, x) <= TOL * 5  # five round trips
    if batch > 1:
        got = last_fwd.cpu().numpy().view(np.complex64).reshape(batch, n)[:8]
        xs = x.cpu().numpy().view(np.complex64).reshape(batch, n)[:8]
        assert rel_l2(got, oracle.fft_c32(xs)) <= TOL * 5
    else:
        bins = np.sort(w.rng(32, log_n).integers(0, n, size=8))
        got = last_fwd[torch.as_tensor(bins, device=cuda)].cpu().numpy().view(np.complex64).reshape(-1)
        want = oracle.dft_bins(x.cpu().numpy().view(np.complex64).reshape(-1), bins)
        assert rel_l2(got, want) <= TOL * 5


def test_zeta_dependent_chain(lib, oracle, cuda):
    """Config 3 in place (chain steps over 16 L2-sized chunks): zeta, inverse
    zeta, zeta, inverse zeta, zeta on the same buffer without synchronising,
    an ordinary torch kernel (+0) between two of them; bit-exact against the
    oracle's zeta of the input."""
    import torch

    from gpu_util import from_device, to_device

    z = w.zeta_input()
    buf = to_device(z, cuda)
    stream = torch.cuda.current_stream().cuda_stream
    n = 1 << w.ZETA_LOG_N

    def t(inverse):
        return cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[n],
                            batch=w.ZETA_BATCH, inverse=inverse, in_place=True)

    with cb.Plan(lib, t(False), stream=stream) as fwd, cb.Plan(lib, t(True), stream=stream) as inv:
        for i in range(5):
            (fwd if i % 2 == 0 else inv).execute(buf.data_ptr(), buf.data_ptr())
            if i == 2:
                buf.add_(0)
        torch.cuda.synchronize()
    assert np.array_equal(from_device(buf, z.dtype, z.shape), oracle.zeta(z))
