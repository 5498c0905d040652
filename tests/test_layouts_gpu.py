"""Strided and padded rank-one layouts on the GPU through the C ABI: the plan
gathers the input layout into a packed workspace buffer, runs the packed
passes there and scatters into the output layout.  Results equal the oracle
on the logical values (bit-exact for zeta / NTT), and output padding keeps its
sentinel."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def layout_view(buf, n, batch, stride, batch_stride):
    """Indices of logical element (b, i) in a flat buffer."""
    b = np.arange(batch)[:, None]
    i = np.arange(n)[None, :]
    return b * batch_stride + i * stride


def run_layout(lib, t, logical, sentinel, cuda):
    """Place `logical` (batch, n) in t's input layout, execute, return the
    logical output and the raw output buffer (host)."""
    from gpu_util import stream_ptr

    n, batch = t.extents[0], t.batch
    dtype = logical.dtype
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        esz = dtype.itemsize
        in_span, out_span = plan.input_size() // esz, plan.output_size() // esz
        host_in = np.full(in_span, sentinel, dtype=dtype)
        host_in[layout_view(host_in, n, batch, t.input_strides[0], t.input_batch_stride)] = logical
        din = torch.from_numpy(host_in.view(np.uint8).copy()).to(cuda)
        if t.in_place:
            dout = din
        else:
            dout = torch.from_numpy(np.full(out_span, sentinel, dtype=dtype).view(np.uint8).copy()).to(cuda)
        ws = None
        if plan.workspace_size():
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
            plan.set_workspace(ws.data_ptr(), ws.numel())
        assert plan.mapping_json().find('"staged_layout":true') >= 0
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        raw = dout.cpu().numpy().view(dtype)
    idx = layout_view(raw, n, batch, t.output_strides[0], t.output_batch_stride)
    return raw[idx], raw, idx


def padding_untouched(raw, idx, sentinel, equal=np.array_equal):
    mask = np.ones(raw.shape, dtype=bool)
    mask[idx.reshape(-1)] = False
    return equal(raw[mask], np.full(mask.sum(), sentinel, dtype=raw.dtype))


@pytest.mark.parametrize("n", [64, 4096, 1 << 15])
def test_fft_strided_input_padded_output(lib, oracle, cuda, n):
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=3,
                     input_strides=[2], output_strides=[1], input_batch_stride=2 * n + 5, output_batch_stride=n + 8)
    x = w.fft_input(n, 3, seed=n)
    got, raw, idx = run_layout(lib, t, x, np.complex64(7 + 7j), cuda)
    assert rel_l2(got, oracle.fft_c32(x)) <= 2e-6
    assert padding_untouched(raw, idx, np.complex64(7 + 7j))


def test_fft_column_layout_with_bit_reversed_output(lib, oracle, cuda):
    """Batches as columns of a row-major N x 6 matrix (not a power-of-two batch,
    so not the native interleaved path), output bit-reversed and packed."""
    n, batch = 256, 6
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=batch,
                     input_strides=[batch], output_strides=[1], input_batch_stride=1, output_batch_stride=n,
                     output_orders=[cb.LogicalOrder.BIT_REVERSED])
    x = w.fft_input(n, batch, seed=2)
    got, _, _ = run_layout(lib, t, x, np.complex64(0), cuda)
    rev = np.array([int(format(i, "08b")[::-1], 2) for i in range(n)])
    assert rel_l2(got, oracle.fft_c32(x)[:, rev]) <= 2e-6


def test_fwht_fp32_padded_rows_in_place(lib, oracle, cuda):
    n, batch = 1024, 5
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[n],
                     batch=batch, input_strides=[1], output_strides=[1], input_batch_stride=n + 16,
                     output_batch_stride=n + 16, in_place=True)
    x = w.rng(3).uniform(-1, 1, size=(batch, n)).astype(np.float32)
    got, raw, idx = run_layout(lib, t, x, np.float32(-3.5), cuda)
    assert rel_l2(got, oracle.fwht_f32(x, normalize=False)) <= 1e-6
    assert padding_untouched(raw, idx, np.float32(-3.5))


def test_bf16_fwht_strided(lib, oracle, cuda):
    n, batch = 4096, 4
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[n],
                     batch=batch, output_scale=1 / 64, output_rounding=cb.OutputRounding.FINAL_STORAGE,
                     input_strides=[3], output_strides=[1], input_batch_stride=3 * n, output_batch_stride=n)
    bits = w.fwht_input_bits(batch, n, seed=4)
    got, _, _ = run_layout(lib, t, bits, np.uint16(0), cuda)
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(w.bf16_bits_to_f32(got), w.bf16_bits_to_f32(want)) <= 4e-3


@pytest.mark.parametrize("op", [cb.Operator.SUBSET_ZETA, cb.Operator.SUPERSET_ZETA])
def test_zeta_strided_both_sides(lib, oracle, cuda, op):
    n, batch = 1 << 14, 3
    t = cb.Transform(op=op, storage=cb.DataType.UINT32, extents=[n], batch=batch, input_strides=[2],
                     output_strides=[3], input_batch_stride=2 * n + 1, output_batch_stride=3 * n + 7)
    z = w.zeta_input(14, batch, seed=6)
    got, raw, idx = run_layout(lib, t, z, np.uint32(0xDEADBEEF), cuda)
    assert np.array_equal(got, oracle.zeta(z, superset=op == cb.Operator.SUPERSET_ZETA))
    assert padding_untouched(raw, idx, np.uint32(0xDEADBEEF))


@pytest.mark.parametrize("n", [256, 1 << 16])
def test_ntt_strided(lib, oracle, cuda, n):
    q = 576460756061519873
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[n], batch=2, modulus=q,
                     input_strides=[2], output_strides=[1], input_batch_stride=2 * n, output_batch_stride=n + 3)
    x = w.rng(7).integers(0, q, size=(2, n), dtype=np.uint64)
    got, raw, idx = run_layout(lib, t, x, np.uint64(12345), cuda)
    assert np.array_equal(got, oracle.ntt_cyclic(x, q))
    assert padding_untouched(raw, idx, np.uint64(12345))


# ---- zero-extended embedding (non-power-of-two logical lengths) ---------------------
def run_sides(lib, t, x, out_len, out_dtype, cuda):
    from gpu_util import from_device, stream_ptr, to_device

    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        din = to_device(x, cuda)
        assert plan.input_size() == din.numel()
        dout = torch.empty(plan.output_size(), dtype=torch.uint8, device=cuda)
        ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        return from_device(dout, out_dtype, (t.batch, out_len)), plan.algorithm_name()


def test_zero_extended_fft_forward_and_inverse(lib, oracle, cuda):
    n, p = 1000, 1024
    x = w.fft_input(n, 3, seed=10)
    t = cb.Transform(op=cb.Operator.FFT, extents=[n], batch=3, length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    got, name = run_sides(lib, t, x, p, np.complex64, cuda)
    padded = np.zeros((3, p), dtype=np.complex64)
    padded[:, :n] = x
    assert name.startswith("zero-extended[")
    assert rel_l2(got, oracle.fft_c32(padded)) <= 2e-6
    spec = w.fft_input(p, 3, seed=11)
    t = cb.Transform(op=cb.Operator.FFT, extents=[n], batch=3, inverse=True,
                     length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    got, _ = run_sides(lib, t, spec, n, np.complex64, cuda)
    assert rel_l2(got, oracle.fft_c32(spec, inverse=True)[:, :n]) <= 2e-6


def test_zero_extended_fwht_zeta_ntt(lib, oracle, cuda):
    x = w.rng(12).uniform(-1, 1, size=(2, 100)).astype(np.float32)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[100],
                     batch=2, length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    got, _ = run_sides(lib, t, x, 128, np.float32, cuda)
    padded = np.zeros((2, 128), dtype=np.float32)
    padded[:, :100] = x
    assert rel_l2(got, oracle.fwht_f32(padded, normalize=False)) <= 1e-6
    z = w.rng(13).integers(0, 1 << 20, size=(2, 3000), dtype=np.uint32)
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[3000], batch=2,
                     length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    got, _ = run_sides(lib, t, z, 4096, np.uint32, cuda)
    zp = np.zeros((2, 4096), dtype=np.uint32)
    zp[:, :3000] = z
    assert np.array_equal(got, oracle.zeta(zp))
    q = 998244353
    v = w.rng(14).integers(0, q, size=(2, 1000), dtype=np.uint64)
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[1000], batch=2, modulus=q,
                     length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING)
    got, _ = run_sides(lib, t, v, 1024, np.uint64, cuda)
    vp = np.zeros((2, 1024), dtype=np.uint64)
    vp[:, :1000] = v
    assert np.array_equal(got, oracle.ntt_cyclic(vp, q))


def test_reference_strided_embedding_fwht(lib, cuda):
    """reference tests/test_c_api.c:791-841: a 6-point FP32 FWHT zero-extended
    to 8 points, written with output stride 2 into 15 floats."""
    from gpu_util import stream_ptr

    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[6],
                     batch=1, length_mode=cb.LengthMode.ZERO_EXTENDED_EMBEDDING, input_strides=[1],
                     output_strides=[2], input_batch_stride=6, output_batch_stride=15)
    expected = np.array([1, 2, 3, 4, 5, 6, 0, 0], dtype=np.float64)
    width = 1
    while width < 8:
        for base in range(0, 8, 2 * width):
            for o in range(width):
                a, b = expected[base + o], expected[base + o + width]
                expected[base + o], expected[base + o + width] = a + b, a - b
        width *= 2
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        assert plan.output_size() == 15 * 4
        din = torch.arange(1, 7, dtype=torch.float32, device=cuda)
        dout = torch.zeros(15, dtype=torch.float32, device=cuda)
        ws = torch.empty(max(plan.workspace_size(), 16), dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        got = dout.cpu().numpy()
    assert np.abs(got[0::2] - expected).max() <= 1e-5


@pytest.mark.parametrize("side", ["strided_in", "strided_out"])
@pytest.mark.parametrize("op", ["fft", "fwht", "zeta", "ntt", "ntt_rev"])
def test_one_packed_side_skips_its_copy(lib, oracle, cuda, side, op):
    """Out of place with one packed side: the core reads the packed input (or
    writes the packed output) directly; results and padding as with both
    sides staged."""
    n, batch = 4096, 3
    strided = dict(input_strides=[2], input_batch_stride=2 * n + 1, output_strides=[1], output_batch_stride=n) \
        if side == "strided_in" else \
        dict(input_strides=[1], input_batch_stride=n, output_strides=[3], output_batch_stride=3 * n + 5)
    q = 576460756061519873
    if op == "fft":
        t = cb.Transform(op=cb.Operator.FFT, extents=[n], batch=batch, **strided)
        x = w.fft_input(n, batch, seed=41)
        want, sentinel = oracle.fft_c32(x), np.complex64(5 - 5j)
    elif op == "fwht":
        t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[n],
                         batch=batch, **strided)
        x = w.rng(42).uniform(-1, 1, size=(batch, n)).astype(np.float32)
        want, sentinel = oracle.fwht_f32(x, normalize=False), np.float32(-9)
    elif op == "zeta":
        t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[n], batch=batch, **strided)
        x = w.zeta_input(12, batch, seed=43)
        want, sentinel = oracle.zeta(x), np.uint32(0xCAFEBABE)
    else:
        orders = dict(output_orders=[cb.LogicalOrder.BIT_REVERSED]) if op == "ntt_rev" else {}
        t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=[n], batch=batch, modulus=q,
                         **orders, **strided)
        x = w.rng(44).integers(0, q, size=(batch, n), dtype=np.uint64)
        want, sentinel = oracle.ntt_cyclic(x, q), np.uint64(31337)
        if op == "ntt_rev":
            want = want[:, [int(format(i, "012b")[::-1], 2) for i in range(n)]]
    got, raw, idx = run_layout(lib, t, x, sentinel, cuda)
    if op == "fft":
        assert rel_l2(got, want) <= 2e-6
    elif op == "fwht":
        assert rel_l2(got, want) <= 1e-6
    else:
        assert np.array_equal(got, want)
    assert padding_untouched(raw, idx, sentinel)
