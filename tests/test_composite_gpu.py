"""Rank-two and rank-three transforms on the GPU through the C ABI (composite
plans of rank-one children): FFT and NTT against the oracle applied along
every axis, FWHT and zeta against the oracle on the flattened index, and the
reference C test's rank-three FWHT known answer."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def run_nd(lib, t, x, cuda, sentinel=0):
    """x: (batch, *extents) logical values placed in t's input layout."""
    from gpu_util import stream_ptr

    dims = len(t.extents)
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        esz = x.dtype.itemsize
        istr = t.input_strides or list(np.cumprod([1] + t.extents[::-1][:-1])[::-1])
        ostr = t.output_strides or istr
        vol = int(np.prod(t.extents))
        ibs = t.input_batch_stride or vol
        obs = t.output_batch_stride or vol
        host = np.full(plan.input_size() // esz, sentinel, dtype=x.dtype)
        grids = np.indices((t.batch, *t.extents)).reshape(dims + 1, -1)
        off_in = grids[0] * ibs + sum(grids[k + 1] * istr[k] for k in range(dims))
        off_out = grids[0] * obs + sum(grids[k + 1] * ostr[k] for k in range(dims))
        host[off_in] = x.reshape(-1)
        din = torch.from_numpy(host.view(np.uint8).copy()).to(cuda)
        dout = din if t.in_place else torch.zeros(plan.output_size(), dtype=torch.uint8, device=cuda)
        ws = None
        if plan.workspace_size():
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
            plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        raw = dout.cpu().numpy().view(x.dtype)
        return raw[off_out].reshape(x.shape), plan.algorithm_name()


def along_axes(fn, x):
    """Apply a rank-one batched transform (rows of the last axis) along every
    transformed axis of x (batch, *extents)."""
    y = x
    for axis in range(1, x.ndim):
        moved = np.moveaxis(y, axis, -1)
        shape = moved.shape
        out = fn(np.ascontiguousarray(moved).reshape(-1, shape[-1])).reshape(shape)
        y = np.moveaxis(out, -1, axis)
    return y


def test_rank_three_fwht_known_answer(lib, cuda):
    """tests/test_c_api.c:698 of the reference: FWHT of 1..8 as 2 x 2 x 2."""
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=[2, 2, 2])
    got, name = run_nd(lib, t, np.arange(1, 9, dtype=np.float32).reshape(1, 2, 2, 2), cuda)
    assert name.startswith("composite[flat:")
    assert np.array_equal(got.reshape(-1), np.array([36, -4, -8, 0, -16, 0, 0, 0], dtype=np.float32))


@pytest.mark.parametrize("extents, batch", [([64, 128], 3), ([8, 16, 32], 2), ([4, 1 << 14], 1), ([2, 4096], 2)])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft_composite(lib, oracle, cuda, extents, batch, inverse):
    vol = int(np.prod(extents))
    x = w.fft_input(vol, batch, seed=vol).reshape(batch, *extents)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=extents, batch=batch,
                     inverse=inverse, normalize_inverse=True)
    got, name = run_nd(lib, t, x, cuda)
    want = along_axes(lambda r: oracle.fft_c32(r, inverse=inverse, normalize=True), x)
    assert name.startswith("composite")
    assert rel_l2(got, want) <= 2e-6, name


def test_fft_composite_padded_layout_in_place(lib, oracle, cuda):
    extents, batch = [32, 64], 2
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=extents, batch=batch,
                     input_strides=[80, 1], output_strides=[80, 1], input_batch_stride=32 * 80 + 16,
                     output_batch_stride=32 * 80 + 16, in_place=True)
    x = w.fft_input(2048, batch, seed=3).reshape(batch, *extents)
    got, _ = run_nd(lib, t, x, cuda, sentinel=np.complex64(1 + 2j))
    assert rel_l2(got, along_axes(lambda r: oracle.fft_c32(r), x)) <= 2e-6


@pytest.mark.parametrize("inverse", [False, True])
def test_ntt_composite(lib, oracle, cuda, inverse):
    q = 998244353
    extents, batch = [16, 256], 2
    x = w.rng(5).integers(0, q, size=(batch, *extents), dtype=np.uint64)
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=extents, batch=batch, modulus=q,
                     inverse=inverse)
    got, _ = run_nd(lib, t, x, cuda)
    assert np.array_equal(got, along_axes(lambda r: oracle.ntt_cyclic(r, q, inverse), x))


def test_zeta_and_fwht_composite(lib, oracle, cuda):
    z = w.zeta_input(12, 2, seed=7).reshape(2, 64, 64)
    t = cb.Transform(op=cb.Operator.SUBSET_ZETA, storage=cb.DataType.UINT32, extents=[64, 64], batch=2,
                     input_strides=[128, 2], output_strides=[64, 1], input_batch_stride=64 * 128,
                     output_batch_stride=4096)
    got, name = run_nd(lib, t, z, cuda)
    assert np.array_equal(got.reshape(2, -1), oracle.zeta(z.reshape(2, -1)))
    bits = w.fwht_input_bits(4, 4096, seed=8)
    t = cb.Transform(op=cb.Operator.FWHT, storage=cb.DataType.BF16, compute=cb.ComputeType.FP32, extents=[64, 64],
                     batch=4, output_scale=1 / 64, output_rounding=cb.OutputRounding.FINAL_STORAGE)
    got, name = run_nd(lib, t, bits.reshape(4, 64, 64), cuda)
    assert name.startswith("composite[flat:")
    want = oracle.fwht_bf16_final(bits, 1 / 64)
    assert rel_l2(w.bf16_bits_to_f32(got.reshape(4, -1)), w.bf16_bits_to_f32(want)) <= 4e-3


def test_legacy_real_fft_adapters(lib, oracle, cuda):
    """cubutterflyPackRealFp32 and cubutterflyExpandHermitianFp32 (reference
    src/real_fft_adapter.cu): real input -> complex (scaled) -> rank-two FFT
    -> half spectrum -> full spectrum rebuilt from Hermitian symmetry."""
    import ctypes as ct

    from gpu_util import stream_ptr

    dll = lib._dll
    dll.cubutterflyPackRealFp32.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_size_t, ct.c_float, ct.c_uint64]
    dll.cubutterflyExpandHermitianFp32.argtypes = [ct.c_void_p, ct.c_void_p, ct.c_uint32, ct.c_uint32, ct.c_size_t,
                                                   ct.c_uint64]
    batch, h, wd = 2, 16, 32
    real = w.rng(9).uniform(-1, 1, size=(batch, h, wd)).astype(np.float32)
    din = torch.from_numpy(real.copy()).to(cuda)
    packed = torch.empty((batch, h, wd, 2), dtype=torch.float32, device=cuda)
    assert dll.cubutterflyPackRealFp32(din.data_ptr(), packed.data_ptr(), real.size, 0.5, stream_ptr()) == 0
    torch.cuda.synchronize()
    got = packed.cpu().numpy()
    assert np.array_equal(got[..., 0], real * np.float32(0.5)) and not got[..., 1].any()
    assert dll.cubutterflyPackRealFp32(None, packed.data_ptr(), 4, 1.0, stream_ptr()) == 1

    x = (real * np.float32(0.5)).astype(np.complex64)
    spectrum = along_axes(lambda r: oracle.fft_c32(r), x)
    half = np.ascontiguousarray(spectrum[..., : wd // 2 + 1])
    dh = torch.from_numpy(half.view(np.float32).copy()).to(cuda)
    full = torch.empty((batch, h, wd, 2), dtype=torch.float32, device=cuda)
    assert dll.cubutterflyExpandHermitianFp32(dh.data_ptr(), full.data_ptr(), h, wd, batch, stream_ptr()) == 0
    torch.cuda.synchronize()
    rebuilt = full.cpu().numpy().view(np.complex64).reshape(batch, h, wd)
    assert rel_l2(rebuilt, spectrum) <= 1e-6


@pytest.mark.parametrize("extents, batch", [([128, 128], 1), ([32, 32, 32], 4), ([64, 64, 64], 2)])
def test_xd_uint32_ntt_measure(lib, oracle, cuda, extents, batch):
    """reference tests/test_c_api.c:298-330: rank-two and rank-three uint32 NTTs
    mod 257 in xD execution mode with the MEASURE policy plan under an
    "xd[" algorithm name; results equal the oracle along every axis."""
    q = 257
    x = w.rng(80, sum(extents)).integers(0, q, size=(batch, *extents), dtype=np.uint32)
    for inverse in (False, True):
        t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32, extents=extents, batch=batch, modulus=q,
                         word_bits=32, inverse=inverse, execution_mode=cb.ExecutionMode.XD)
        got, name = run_nd_opts(lib, t, x, cuda, cb.PlanOptions(policy=cb.AlgorithmPolicy.MEASURE))
        assert name.startswith("xd["), name
        want = along_axes(lambda r: oracle.ntt_cyclic(r.astype(np.uint64), q, inverse), x.astype(np.uint64))
        assert np.array_equal(got.astype(np.uint64), want), (extents, inverse)


def run_nd_opts(lib, t, x, cuda, options):
    from gpu_util import stream_ptr

    with cb.Plan(lib, t, options=options, stream=stream_ptr()) as plan:
        din = torch.from_numpy(np.ascontiguousarray(x).view(np.uint8).reshape(-1).copy()).to(cuda)
        dout = torch.zeros(plan.output_size(), dtype=torch.uint8, device=cuda)
        if plan.workspace_size():
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
            plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        return dout.cpu().numpy().view(x.dtype).reshape(x.shape), plan.algorithm_name()


@pytest.mark.parametrize("word_bits", [32, 64])
def test_reference_algorithm_name_runs_this_builds_mapping(lib, oracle, cuda, word_bits):
    """reference tests/test_c_api.c:920-975 asks for its "ntt-shared-iterative"
    kernels by name: here the name is accepted, this build's mapping runs, and
    the natural and bit-reversed output layouts agree up to the permutation."""
    q = 998244353 if word_bits == 32 else 576460756061519873
    dt = np.uint32 if word_bits == 32 else np.uint64
    x = (np.arange(16, dtype=np.uint64) * 17 + 3).astype(dt).reshape(2, 8)
    outs = []
    for order in (cb.NttLayout.NATURAL, cb.NttLayout.BIT_REVERSED):
        t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32 if word_bits == 32 else cb.DataType.UINT64,
                         extents=[8], batch=2, modulus=q, word_bits=word_bits, output_order=order)
        got, _ = run_nd_opts(lib, t, x, cuda, cb.PlanOptions(mapping="ntt-shared-iterative"))
        outs.append(got)
    rev = [int(format(i, "03b")[::-1], 2) for i in range(8)]
    assert np.array_equal(outs[1], outs[0][:, rev])
    assert np.array_equal(outs[0].astype(np.uint64), oracle.ntt_cyclic(x.astype(np.uint64), q))


@pytest.mark.parametrize("extents, batch, in_place", [([1024, 1024], 2, False), ([256, 64, 64], 2, False),
                                                     ([64, 128], 3, True), ([16, 8192], 1, False)])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft_composite_direct(lib, oracle, cuda, extents, batch, in_place, inverse):
    """Packed power-of-two FFTs whose outer axes qualify as interleaved batches
    run without gather, transposes or scatter: the innermost axis from the
    input into the output, each outer axis in place as blocks of interleaved
    transforms."""
    vol = int(np.prod(extents))
    x = w.fft_input(vol, batch, seed=vol + 5).reshape(batch, *extents)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=extents, batch=batch,
                     inverse=inverse, normalize_inverse=True, in_place=in_place)
    got, name = run_nd(lib, t, x, cuda)
    assert name.startswith("composite-direct["), name
    want = along_axes(lambda r: oracle.fft_c32(r, inverse=inverse, normalize=True), x)
    assert rel_l2(got, want) <= 2e-6, name
