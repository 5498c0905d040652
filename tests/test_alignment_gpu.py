"""Element-aligned caller buffers (the reference's contract: any element
pointer of a device buffer, e.g. a view at an odd offset), through the C ABI.

Complex FFTs and NTTs move whole elements in every kernel; FWHT and zeta run
their element-granular kernels when a pointer is not 16-byte aligned.  Each
case is checked against the oracle at the usual tolerance (bit-exact for
integers) with input and output at odd element offsets, out of place and in
place; pointers below element alignment and stage-storage plans at odd
offsets are rejected."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w
from gpu_util import stream_ptr

pytestmark = pytest.mark.gpu


def run_offset(lib, t, x, cuda, in_off, out_off, itemsize):
    """Execute `t` on host array x placed `in_off` elements into a device
    buffer, writing `out_off` elements into another (the same buffer when in
    place); returns the output as x's dtype and shape."""
    nbytes = x.nbytes
    raw_in = np.zeros(nbytes + 64, dtype=np.uint8)
    raw_in[in_off * itemsize:in_off * itemsize + nbytes] = np.ascontiguousarray(x).view(np.uint8).reshape(-1)
    din = torch.from_numpy(raw_in).to(cuda)
    dout = din if t.in_place else torch.zeros(nbytes + 64, dtype=torch.uint8, device=cuda)
    off = in_off if t.in_place else out_off
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        ws = torch.empty(max(plan.workspace_size(), 16), dtype=torch.uint8, device=cuda)
        if plan.workspace_size():
            plan.set_workspace(ws.data_ptr(), plan.workspace_size())
        plan.execute(din.data_ptr() + in_off * itemsize, dout.data_ptr() + off * itemsize)
        torch.cuda.synchronize()
        name = plan.algorithm_name()
    got = dout.cpu().numpy()[off * itemsize:off * itemsize + nbytes].copy()
    return got.view(x.dtype).reshape(x.shape), name


@pytest.mark.parametrize("in_off, out_off, in_place", [(1, 3, False), (5, 0, False), (3, 3, True)])
def test_fwht_bf16_odd_offsets(lib, oracle, cuda, in_off, out_off, in_place):
    """Config 1's operator on a bf16 view at an odd element offset (2-byte aligned)."""
    bits = w.fwht_input_bits(64, 4096, seed=8)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[4096],
                     batch=64, output_scale=1 / 64, output_rounding=cb.OutputRounding.FINAL_STORAGE,
                     in_place=in_place)
    got, _ = run_offset(lib, t, bits, cuda, in_off, out_off, 2)
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(w.bf16_bits_to_f32(got), w.bf16_bits_to_f32(want)) <= 4e-3
    assert np.mean(got == want) > 0.99


@pytest.mark.parametrize("n", [2, 128, 1 << 14])
def test_fwht_f32_odd_offsets(lib, oracle, cuda, n):
    x = w.rng(70, n).standard_normal((5, n)).astype(np.float32)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[n], batch=5,
                     inverse=True, normalize_inverse=True)
    got, _ = run_offset(lib, t, x, cuda, 1, 2, 4)
    assert rel_l2(got, oracle.fwht_f32(x, inverse=True, normalize=True)) <= 1e-6


@pytest.mark.parametrize("log_n, superset, inverse, in_place", [(12, False, False, False), (14, True, True, True),
                                                               (16, False, True, False), (20, True, False, True)])
def test_zeta_odd_offsets(lib, oracle, cuda, log_n, superset, inverse, in_place):
    z = w.zeta_input(log_n, 3, seed=log_n)
    t = cb.Transform(op=cb.Operator.SUPERSET_ZETA if superset else cb.Operator.SUBSET_ZETA,
                     storage=cb.DataType.UINT32, extents=[1 << log_n], batch=3, inverse=inverse, in_place=in_place)
    got, _ = run_offset(lib, t, z, cuda, 1, 3, 4)
    assert np.array_equal(got, oracle.zeta(z, superset=superset, inverse=inverse))


def test_zeta_u64_odd_offset(lib, oracle, cuda):
    z = w.rng(71).integers(0, 2**63, size=(2, 1 << 15), dtype=np.uint64)
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT64, extents=[1 << 15], batch=2)
    got, _ = run_offset(lib, t, z, cuda, 1, 1, 8)
    assert np.array_equal(got, oracle.zeta(z))


@pytest.mark.parametrize("log_n, batch", [(12, 64), (20, 2), (5, 9)])
def test_fft_c64_odd_offsets(lib, oracle, cuda, log_n, batch):
    """Complex fp32 at odd complex offsets (8-byte aligned): the local FFT takes
    its float2 kernel, the global passes move float2 already."""
    x = w.fft_input(1 << log_n, batch, seed=log_n)
    t = cb.Transform(op=cb.Operator.FFT, extents=[1 << log_n], batch=batch)
    got, _ = run_offset(lib, t, x, cuda, 1, 3, 8)
    assert rel_l2(got, oracle.fft_c32(x)) <= 2e-6


def test_ntt_u64_odd_offset(lib, oracle, cuda):
    q = 576460756061519873
    x = w.rng(72).integers(0, q, size=(4, 1 << 12), dtype=np.uint64)
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[1 << 12], batch=4, modulus=q)
    got, _ = run_offset(lib, t, x, cuda, 1, 1, 8)
    assert np.array_equal(got, oracle.ntt_cyclic(x, q))


def test_below_element_alignment_and_stage_storage_are_rejected(lib, cuda):
    buf = torch.zeros(1 << 16, dtype=torch.uint8, device=cuda)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[256],
                     batch=4, output_rounding=cb.OutputRounding.FINAL_STORAGE)
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        with pytest.raises(cb.Error) as e:
            plan.execute(buf.data_ptr() + 1, buf.data_ptr() + 4096)  # 1 byte: not a bf16 element
        assert e.value.status == cb.Status.INVALID_VALUE
    s = cb.Transform(op=cb.Operator.STRUCTURED_2X2, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32,
                     extents=[256], batch=4, stage_matrices=[[(1.0, 0.5, -0.5, 1.0)]])
    with cb.Plan(lib, s, stream=stream_ptr()) as plan:
        with pytest.raises(cb.Error) as e:
            plan.execute(buf.data_ptr() + 4, buf.data_ptr() + 8192)
        assert e.value.status == cb.Status.NOT_SUPPORTED
