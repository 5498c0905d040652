"""Non-power-of-two complex FFTs on the GPU through the C ABI: Bluestein
convolutions over the library's power-of-two FFTs (reference
src/bluestein_fft.cu).  Checked against the oracle's direct long-double DFT:
relative L2 <= 2e-6 for complex FP32 storage (the FP32 FFT bar), <= 1e-12 for
complex FP64; plus the reference C test's 5-point known answer."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu

C32, C64 = cb.DataType.COMPLEX_FP32, cb.DataType.COMPLEX_FP64


def transform(extents, batch, storage=C32, **kw):
    compute = cb.ComputeType.FP64 if storage == C64 else cb.ComputeType.FP32
    return cb.Transform(op=cb.Operator.FFT, storage=storage, compute=compute, extents=extents, batch=batch, **kw)


def signal(shape, seed, dtype=np.complex64):
    g = w.rng(60, seed)
    return (g.uniform(-1, 1, size=shape) + 1j * g.uniform(-1, 1, size=shape)).astype(dtype)


def test_reference_five_point_known_answer(lib, cuda):
    """reference tests/test_c_api.c:49-108: the 5-point FFT of an impulse at
    index 1 is exp(-2 pi i k / 5) (abs 2e-5), the plan's physical extent is the
    16-point convolution, and the normalised inverse recovers the impulse."""
    from gpu_util import run, stream_ptr

    x = np.zeros((1, 5), dtype=np.complex64)
    x[0, 1] = 1
    t = transform([5], 1)
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        assert plan.physical_extents(1) == [16]
        assert plan.algorithm_name().startswith("bluestein[16:")
    y, _ = run(lib, t, x, cuda)
    k = np.arange(5)
    assert np.abs(y[0] - np.exp(-2j * np.pi * k / 5)).max() <= 2e-5
    back, _ = run(lib, transform([5], 1, inverse=True, normalize_inverse=True), y, cuda)
    assert np.abs(back - x).max() <= 2e-5


@pytest.mark.parametrize("n", [3, 5, 6, 12, 100, 1000, 4095, 12289])
@pytest.mark.parametrize("inverse", [False, True])
def test_fp32_against_direct_dft(lib, oracle, cuda, n, inverse):
    from gpu_util import run

    x = signal((3, n), n)
    got, name = run(lib, transform([n], 3, inverse=inverse, normalize_inverse=True), x, cuda)
    want = oracle.dft(x, inverse=inverse, normalize=True)
    assert name.startswith("bluestein[")
    assert rel_l2(got, want) <= 2e-6, (name, rel_l2(got, want))


@pytest.mark.parametrize("n", [7, 1000, 3 * 4096])
def test_fp64_against_direct_dft(lib, oracle, cuda, n):
    from gpu_util import run

    x = signal((2, n), n + 1, np.complex128)
    for inverse in (False, True):
        got, _ = run(lib, transform([n], 2, C64, inverse=inverse, normalize_inverse=False), x, cuda)
        assert rel_l2(got, oracle.dft(x, inverse=inverse, normalize=False)) <= 1e-12


def test_strided_layout_and_in_place(lib, oracle, cuda):
    """Any rank-one layout: the pack reads the input layout and the unpack
    writes the output layout directly; padding keeps its sentinel.  In place
    gives the same result."""
    import test_layouts_gpu as tl
    from gpu_util import run, stream_ptr

    n, batch = 300, 4
    x = signal((batch, n), 7)
    t = transform([n], batch, input_strides=[2], output_strides=[1], input_batch_stride=2 * n + 3,
                  output_batch_stride=n + 5)
    sentinel = np.complex64(3 + 4j)
    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        host_in = np.full(plan.input_size() // 8, sentinel, dtype=np.complex64)
        idx_in = tl.layout_view(host_in, n, batch, 2, 2 * n + 3)
        host_in[idx_in] = x
        din = torch.from_numpy(host_in.view(np.uint8).copy()).to(cuda)
        dout = torch.from_numpy(np.full(plan.output_size() // 8, sentinel, dtype=np.complex64).view(np.uint8)
                                .copy()).to(cuda)
        ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        raw = dout.cpu().numpy().view(np.complex64)
    idx = tl.layout_view(raw, n, batch, 1, n + 5)
    assert rel_l2(raw[idx], oracle.dft(x)) <= 2e-6
    assert tl.padding_untouched(raw, idx, sentinel)
    got, _ = run(lib, transform([n], batch, in_place=True), x, cuda)
    assert rel_l2(got, oracle.dft(x)) <= 2e-6


@pytest.mark.parametrize("extents", [[6, 10], [12, 64], [100, 3]])
def test_rank_two_against_direct_dft(lib, oracle, cuda, extents):
    from test_composite_gpu import along_axes, run_nd

    x = signal((2, *extents), sum(extents))
    got, name = run_nd(lib, transform(extents, 2), x, cuda)
    want = along_axes(lambda r: oracle.dft(r), x.astype(np.complex128))
    assert name.startswith("composite[") and "bluestein" in name
    assert rel_l2(got, want) <= 2e-6
    with cb.Plan(lib, transform(extents, 2)) as plan:
        assert plan.physical_extents(2) == [e if (e & (e - 1)) == 0 else 1 << (2 * e - 2).bit_length()
                                            for e in extents]


# ---- NTT of non-power-of-two lengths (u64 words), bit-exact ---------------------
DEFAULT_Q = 1152921504606584833  # q - 1 = 2^18 3^2 7^2 43 127 337 5419


def ntt_transform(n, batch, inverse=False, q=DEFAULT_Q, **kw):
    return cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT64, extents=n if isinstance(n, list) else [n],
                        batch=batch, modulus=q, inverse=inverse, **kw)


def test_ntt_reference_round_trip(lib, oracle, cuda):
    """reference tests/test_c_api.c:332-383: {7, 11, 19} under the default
    modulus, forward then inverse."""
    from gpu_util import run

    x = np.array([[7, 11, 19]], dtype=np.uint64)
    y, name = run(lib, ntt_transform(3, 1), x, cuda)
    assert name.startswith("bluestein-ntt[8:")
    assert np.array_equal(y, oracle.ntt_any(x, DEFAULT_Q))
    back, _ = run(lib, ntt_transform(3, 1, inverse=True), y, cuda)
    assert np.array_equal(back, x)


@pytest.mark.parametrize("n", [3, 7, 12, 63, 127, 903, 5419])
def test_ntt_against_oracle(lib, oracle, cuda, n):
    """Full 64-bit input words (reduced on load), forward and inverse."""
    from gpu_util import run

    x = w.rng(71, n).integers(0, 2**64, size=(3, n), dtype=np.uint64)
    for inverse in (False, True):
        got, _ = run(lib, ntt_transform(n, 3, inverse), x, cuda)
        assert np.array_equal(got, oracle.ntt_any(x, DEFAULT_Q, inverse)), (n, inverse)


def test_ntt_layouts_rank_two_and_bad_modulus(lib, oracle, cuda):
    from gpu_util import run
    from test_composite_gpu import along_axes, run_nd

    n, batch = 63, 4
    x = w.rng(72).integers(0, DEFAULT_Q, size=(batch, n), dtype=np.uint64)
    got, _ = run(lib, ntt_transform(n, batch, in_place=True), x, cuda)
    assert np.array_equal(got, oracle.ntt_any(x, DEFAULT_Q))
    from test_layouts_gpu import padding_untouched

    t = ntt_transform(n, batch, input_strides=[3], output_strides=[2], input_batch_stride=3 * n + 1,
                      output_batch_stride=2 * n + 5)
    import test_layouts_gpu as tl

    from gpu_util import stream_ptr

    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        host = np.full(plan.input_size() // 8, 99, dtype=np.uint64)
        host[tl.layout_view(host, n, batch, 3, 3 * n + 1)] = x
        din = torch.from_numpy(host.view(np.uint8).copy()).to(cuda)
        dout = torch.from_numpy(np.full(plan.output_size() // 8, 77, dtype=np.uint64).view(np.uint8).copy()).to(cuda)
        ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        raw = dout.cpu().numpy().view(np.uint64)
    idx = tl.layout_view(raw, n, batch, 2, 2 * n + 5)
    assert np.array_equal(raw[idx], oracle.ntt_any(x, DEFAULT_Q))
    assert padding_untouched(raw, idx, np.uint64(77))
    # rank two: 7 x 12, each axis its own length
    x2 = w.rng(73).integers(0, DEFAULT_Q, size=(2, 7, 12), dtype=np.uint64)
    got2, name = run_nd(lib, ntt_transform([7, 12], 2), x2, cuda)
    assert "bluestein-ntt" in name
    assert np.array_equal(got2, along_axes(lambda r: oracle.ntt_any(r, DEFAULT_Q), x2))
    # 2n must divide q - 1: 11 does not divide the default modulus's q - 1
    with pytest.raises(cb.Error) as e:
        cb.Plan(lib, ntt_transform(11, 1))
    assert "2N-th Bluestein root" in str(e.value)
