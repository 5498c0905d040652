"""FFT parity on the GPU through the C ABI: rel L2 <= 2e-6 against the oracle
(reference_fft<Complex32> semantics), plus bit-level checks against the
golden fixtures made by the reference's own compiled oracle."""
import os

import numpy as np
import pytest

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu
TOL = 2e-6  # relative L2, fp32 FFT (north_star)


def fft_transform(n, batch, inverse=False, normalize=True, in_place=False):
    return cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=batch,
                        inverse=inverse, normalize_inverse=normalize, in_place=in_place)


@pytest.mark.parametrize("n", [2, 4, 8, 16, 32, 64, 128, 256, 512, 1024, 2048, 4096, 8192])
def test_fft_forward_sizes(lib, oracle, cuda, n):
    from gpu_util import run

    x = w.fft_input(n, 17, seed=n)
    got, name = run(lib, fft_transform(n, 17), x, cuda)
    assert rel_l2(got, oracle.fft_c32(x)) <= TOL, name


@pytest.mark.parametrize("n", [16, 4096, 8192])
@pytest.mark.parametrize("normalize", [False, True])
def test_fft_inverse(lib, oracle, cuda, n, normalize):
    from gpu_util import run

    x = w.fft_input(n, 5, seed=3)
    got, _ = run(lib, fft_transform(n, 5, inverse=True, normalize=normalize), x, cuda)
    assert rel_l2(got, oracle.fft_c32(x, inverse=True, normalize=normalize)) <= TOL


@pytest.mark.parametrize("n", [8, 64, 1024, 4096])
def test_fft_golden(lib, golden, cuda, n):
    from gpu_util import run

    x = golden[f"fft_fwd_{n}_in"]
    got, _ = run(lib, fft_transform(n, x.shape[0]), x, cuda)
    assert rel_l2(got, golden[f"fft_fwd_{n}_out"]) <= TOL


def test_fft_in_place_and_ragged_batch(lib, oracle, cuda):
    from gpu_util import run

    for batch in (1, 3, 129):
        x = w.fft_input(4096, batch, seed=batch)
        got, _ = run(lib, fft_transform(4096, batch, in_place=True), x, cuda)
        assert rel_l2(got, oracle.fft_c32(x)) <= TOL


def test_fft_config0_full_size(lib, oracle, cuda):
    """Config 0: N = 4096, batch 1024, natural in/out, unnormalized."""
    from gpu_util import run

    x = w.fft_input()
    got, name = run(lib, fft_transform(w.FFT_N, w.FFT_BATCH), x, cuda)
    err = rel_l2(got, oracle.fft_c32(x))
    assert err <= TOL, (name, err)


def test_fft_round_trip(lib, cuda):
    from gpu_util import run

    x = w.fft_input(2048, 8, seed=1)
    f, _ = run(lib, fft_transform(2048, 8), x, cuda)
    back, _ = run(lib, fft_transform(2048, 8, inverse=True, normalize=True), f, cuda)
    assert rel_l2(back, x) <= TOL


# ---- multi-pass global FFT (N > 2^13) ----------------------------------------------
@pytest.mark.parametrize("log_n", [14, 15, 16, 18, 20])
def test_fft_multipass_sizes(lib, oracle, cuda, log_n):
    from gpu_util import run

    batch = 3 if log_n <= 16 else 1
    x = w.fft_input(1 << log_n, batch, seed=log_n)
    got, name = run(lib, fft_transform(1 << log_n, batch), x, cuda)
    assert name.startswith("fft-stockham-global"), name
    assert rel_l2(got, oracle.fft_c32(x)) <= TOL, name


@pytest.mark.parametrize("in_place", [False, True])
@pytest.mark.parametrize("log_n", [17, 21])
def test_fft_multipass_inverse_in_place(lib, oracle, cuda, log_n, in_place):
    """Odd and even pass counts (2 and 3 passes), with the in-place workspace."""
    from gpu_util import run

    x = w.fft_input(1 << log_n, 2, seed=2)
    got, _ = run(lib, fft_transform(1 << log_n, 2, inverse=True, normalize=True, in_place=in_place), x, cuda)
    assert rel_l2(got, oracle.fft_c32(x, inverse=True, normalize=True)) <= TOL


def test_fft_2_24_spot_bins_and_round_trip(lib, oracle, cuda):
    """Large single transform: direct long-double DFT at 8 bins, plus inverse(forward(x)) == x."""
    from gpu_util import run

    n = 1 << 24
    x = w.fft_input(n, 1, seed=24)
    f, name = run(lib, fft_transform(n, 1), x, cuda)
    bins = w.rng(77).integers(0, n, size=8)
    ref = oracle.dft_bins(x[0], bins)
    assert rel_l2(f[0][bins], ref) <= TOL, name
    back, _ = run(lib, fft_transform(n, 1, inverse=True, normalize=True), f, cuda)
    assert rel_l2(back, x) <= TOL


def interleaved_transform(n, batch, inverse=False, normalize=True, in_place=False):
    """Batches interleaved element-wise: element k of transform b at k * batch + b
    (the columns of a row-major n x batch matrix), through cubutterflySetStrides."""
    return cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=batch,
                        inverse=inverse, normalize_inverse=normalize, in_place=in_place, input_strides=[batch],
                        output_strides=[batch], input_batch_stride=1, output_batch_stride=1)


@pytest.mark.parametrize("n, batch", [(16, 256), (256, 32), (4096, 64), (1 << 15, 16), (1 << 14, 4), (8192, 512), (1024, 4)])
@pytest.mark.parametrize("inverse", [False, True])
def test_fft_interleaved_batches(lib, oracle, cuda, n, batch, inverse):
    from gpu_util import run

    x = w.fft_input(n, batch, seed=n + batch)
    cols = np.ascontiguousarray(x.T)  # (n, batch): transform b is column b
    got, name = run(lib, interleaved_transform(n, batch, inverse=inverse), cols, cuda)
    assert name.startswith("fft-stockham-global"), name
    want = oracle.fft_c32(x, inverse=inverse, normalize=True)
    assert rel_l2(np.ascontiguousarray(got.reshape(n, batch).T), want) <= TOL, name


def test_fft_interleaved_in_place(lib, oracle, cuda):
    from gpu_util import run

    n, batch = 1 << 13, 128
    x = w.fft_input(n, batch, seed=5)
    got, _ = run(lib, interleaved_transform(n, batch, in_place=True), np.ascontiguousarray(x.T), cuda)
    assert rel_l2(np.ascontiguousarray(got.reshape(n, batch).T), oracle.fft_c32(x)) <= TOL


# ---- R2C / C2R (over an N/2-point complex FFT) --------------------------------------
def run_real(lib, t, x, out_shape, out_dtype, cuda):
    import torch

    from gpu_util import from_device, stream_ptr, to_device

    with cb.Plan(lib, t, stream=stream_ptr()) as plan:
        din = to_device(x, cuda)
        assert plan.input_size() == din.numel()
        dout = torch.empty(plan.output_size(), dtype=torch.uint8, device=cuda)
        ws = torch.empty(max(plan.workspace_size(), 1), dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr(), plan.workspace_size())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        return from_device(dout, out_dtype, out_shape), plan.algorithm_name()


@pytest.mark.parametrize("n", [4, 64, 4096, 1 << 15])
@pytest.mark.parametrize("scale", [1.0, 0.5])
def test_r2c(lib, oracle, cuda, n, scale):
    x = w.rng(n).uniform(-1, 1, size=(3, n)).astype(np.float32)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[n], batch=3, fft_type=cb.FftType.R2C,
                     fft_output_scale=scale)
    got, name = run_real(lib, t, x, (3, n // 2 + 1), np.complex64, cuda)
    want = oracle.fft_c32(x.astype(np.complex64))[:, : n // 2 + 1] * np.float32(scale)
    assert name.startswith("fft-r2c[")
    assert rel_l2(got, want) <= TOL, name


@pytest.mark.parametrize("n", [4, 64, 4096, 1 << 15])
@pytest.mark.parametrize("normalize", [True, False])
def test_c2r(lib, oracle, cuda, n, normalize):
    real = w.rng(n + 1).uniform(-1, 1, size=(3, n)).astype(np.float32)
    half = np.ascontiguousarray(oracle.fft_c32(real.astype(np.complex64))[:, : n // 2 + 1])  # Hermitian half
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, extents=[n], batch=3, fft_type=cb.FftType.C2R,
                     inverse=True, normalize_inverse=normalize)
    got, name = run_real(lib, t, half, (3, n), np.float32, cuda)
    full = np.concatenate([half, np.conj(half[:, 1:-1][:, ::-1])], axis=1)
    want = oracle.fft_c32(full, inverse=True, normalize=normalize).real
    assert name.startswith("fft-c2r[")
    assert rel_l2(got, want) <= TOL, name
    if normalize:
        assert rel_l2(got, real) <= TOL  # round trip R2C -> C2R


# ---- complex fp64 FFT (radix 2, bit-identical to reference_fft<Complex64>) -----------
@pytest.mark.parametrize("n", [2, 64, 2048, 1 << 14, 1 << 20])
@pytest.mark.parametrize("inverse, normalize", [(False, False), (True, True), (True, False)])
def test_fft_fp64(lib, oracle, cuda, n, inverse, normalize):
    from gpu_util import run

    x = w.fft_input(n, 3, seed=n).astype(np.complex128)
    x += 1e-9 * w.fft_input(n, 3, seed=n + 1)  # low-order bits beyond fp32
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP64, compute=cb.ComputeType.FP64,
                     extents=[n], batch=3, inverse=inverse, normalize_inverse=normalize)
    got, name = run(lib, t, x, cuda)
    assert name.startswith("fft64-radix2")
    assert np.array_equal(got, oracle.fft_c64(x, inverse=inverse, normalize=normalize)), name


def test_fft_fp64_matches_reference_and_composite(lib, oracle, reference, cuda):
    """Pinned to the reference's own reference_fft<Complex64>; a rank-two fp64
    FFT runs per axis through the composite path."""
    from gpu_util import run

    x = w.fft_input(4096, 2, seed=5).astype(np.complex128)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP64, compute=cb.ComputeType.FP64,
                     extents=[4096], batch=2)
    got, _ = run(lib, t, x, cuda)
    assert np.array_equal(got, reference.fft_c64(x))
    x2 = w.fft_input(32 * 64, 2, seed=6).astype(np.complex128).reshape(2, 32, 64)
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP64, compute=cb.ComputeType.FP64,
                     extents=[32, 64], batch=2)
    got, name = run(lib, t, x2.reshape(2, -1), cuda)
    want = oracle.fft_c64(np.swapaxes(oracle.fft_c64(x2), 1, 2).copy())
    assert rel_l2(got.reshape(2, 32, 64), np.swapaxes(want, 1, 2)) <= 1e-13, name


# ---- config 4: one 2^30-point transform at its stated size -------------------------------
def _rel_l2_dev(a, b, chunk=1 << 26):
    """Relative L2 of two equal-shape device tensors, summed in fp64 over chunks."""
    import torch

    a, b = a.reshape(-1), b.reshape(-1)
    num = den = 0.0
    for i in range(0, a.numel(), chunk):
        x, y = a[i:i + chunk].double(), b[i:i + chunk].double()
        num += float(torch.sum((x - y) ** 2))
        den += float(torch.sum(y * y))
    return (num / den) ** 0.5


def test_fft_config4_2e30_single_gpu(lib, oracle, cuda):
    """Config 4 on one GPU at full size (8 GiB in, 8 GiB out): 16 random bins
    against the oracle's long-double direct DFT, the inverse round trip, and
    every output against this library's fp64 FFT (bit-identical to the
    reference's reference_fft<Complex64> at the sizes the CPU can check)."""
    import torch

    n = 1 << 30
    x = w.torch_fft_input(n, 1, cuda, seed=4).reshape(n, 2)
    stream = torch.cuda.current_stream().cuda_stream

    def planned(t, src):
        with cb.Plan(lib, t, stream=stream) as p:
            ws = torch.empty(max(p.workspace_size(), 16), dtype=torch.uint8, device=cuda)
            if p.workspace_size():
                p.set_workspace(ws.data_ptr(), p.workspace_size())
            dst = torch.empty(p.output_size() // src.element_size(), dtype=src.dtype, device=cuda)
            p.execute(src.data_ptr(), dst.data_ptr())
            torch.cuda.synchronize()
            return dst.reshape(src.shape), p.algorithm_name()

    y, name = planned(fft_transform(n, 1), x)
    bins = np.sort(w.rng(78).integers(0, n, size=16))
    got = y[torch.as_tensor(bins, device=cuda)].cpu().numpy().view(np.complex64).reshape(-1)
    host_x = x.cpu().numpy().view(np.complex64).reshape(-1)
    ref = oracle.dft_bins(host_x, bins)
    del host_x
    assert rel_l2(got, ref) <= TOL, name
    back, _ = planned(fft_transform(n, 1, inverse=True, normalize=True), y)
    assert _rel_l2_dev(back, x) <= TOL
    del back
    t64 = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP64, compute=cb.ComputeType.FP64,
                       extents=[n], batch=1)
    y64, name64 = planned(t64, x.double())
    assert _rel_l2_dev(y, y64) <= TOL, (name, name64)


def test_four_step_2e24_matches_the_reference_fft(cuda, reference):
    """The four-step decomposition (one rank) at 2^24 against the reference's
    own reference_fft<Complex32> (src/butterfly_reference.cpp:392-473),
    compiled unchanged into oracle/_ref."""
    import torch

    from cubutterfly_b200.distributed import FourStepFFT

    n = 1 << 24
    x = w.fft_input(n, 1, seed=124)[0]
    fs = FourStepFFT(n, device=cuda)
    got = fs(torch.from_numpy(x.view(np.float32).reshape(n, 2).copy()).to(cuda))
    torch.cuda.synchronize()
    fs.close()
    got = got.cpu().numpy().view(np.complex64).reshape(-1)
    want = reference.fft_c32(x[None], threads=os.cpu_count() or 1)[0]
    assert rel_l2(got, want) <= TOL


@pytest.mark.parametrize("log_n, mapping", [(24, "fft-l2-blocked[8+6+10]"), (26, "fft-l2-blocked[8+8+10]"),
                                            (28, "fft-l2-blocked[9+9+10]"), (27, "fft-l2-blocked[9+8+10]")])
def test_fft_l2_blocked_plans(lib, oracle, cuda, log_n, mapping):
    """The L2-blocked plan of long transforms (V = 2^10 decimated transforms
    taken 8 at a time through L2, then one combining pass; an EXPLICIT or
    MEASURE choice, not the static default): against the
    Stockham multi-pass plan on the same input, 8 DFT bins against the
    oracle's long-double direct DFT, the normalised inverse round trip, and in
    place; all at rel L2 <= 2e-6."""
    import torch

    n = 1 << log_n
    x = w.torch_fft_input(n, 1, cuda, seed=log_n).reshape(n, 2)
    stream = torch.cuda.current_stream().cuda_stream

    def planned(t, src, options=None):
        with cb.Plan(lib, t, options=options, stream=stream) as p:
            ws = torch.empty(max(p.workspace_size(), 16), dtype=torch.uint8, device=cuda)
            if p.workspace_size():
                p.set_workspace(ws.data_ptr(), p.workspace_size())
            dst = src if t.in_place else torch.empty_like(src)
            p.execute(src.data_ptr(), dst.data_ptr())
            torch.cuda.synchronize()
            return dst, p.algorithm_name()

    opts = cb.PlanOptions(mapping=mapping)
    y, name = planned(fft_transform(n, 1), x, opts)
    assert name.startswith("fft-l2-blocked"), name
    ref, ref_name = planned(fft_transform(n, 1), x, cb.PlanOptions(mapping="8+8+" + "+".join(
        str(p) for p in ([log_n - 16] if log_n - 16 <= 10 else [(log_n - 16) // 2, log_n - 16 - (log_n - 16) // 2]))))
    assert ref_name.startswith("fft-stockham-global"), ref_name
    assert _rel_l2_dev(y, ref) <= TOL, (name, ref_name)
    bins = np.sort(w.rng(79, log_n).integers(0, n, size=8))
    got = y[torch.as_tensor(bins, device=cuda)].cpu().numpy().view(np.complex64).reshape(-1)
    assert rel_l2(got, oracle.dft_bins(x.cpu().numpy().view(np.complex64).reshape(-1), bins)) <= TOL
    back, _ = planned(fft_transform(n, 1, inverse=True, normalize=True), y, opts)
    assert _rel_l2_dev(back, x) <= TOL
    z = x.clone()
    z, _ = planned(fft_transform(n, 1, in_place=True), z, opts)
    assert _rel_l2_dev(z, y) <= TOL


@pytest.mark.parametrize("log_n, mapping", [(26, "fft-l2-chain[8+6+6+6]"), (27, "fft-l2-chain[8+7+6+6]"),
                                            (28, "fft-l2-chain[8+7+7+6]")])
def test_fft_l2_chain_plans(lib, oracle, cuda, log_n, mapping):
    """The L2-chained plan (four Stockham passes run as two chunked pairs, the
    second pass of each chunk reading the first one's output from L2): against
    the Stockham plan on the same input, 8 DFT bins against the oracle's
    long-double direct DFT, the normalised inverse round trip, a batch of two
    transforms, and an in-place request (served by another plan); rel L2 <=
    2e-6."""
    import torch

    n = 1 << log_n
    x = w.torch_fft_input(n, 2, cuda, seed=log_n).reshape(2 * n, 2)
    stream = torch.cuda.current_stream().cuda_stream

    def planned(t, src, options=None):
        with cb.Plan(lib, t, options=options, stream=stream) as p:
            ws = torch.empty(max(p.workspace_size(), 16), dtype=torch.uint8, device=cuda)
            if p.workspace_size():
                p.set_workspace(ws.data_ptr(), p.workspace_size())
            dst = src if t.in_place else torch.empty_like(src)
            p.execute(src.data_ptr(), dst.data_ptr())
            torch.cuda.synchronize()
            return dst, p.algorithm_name()

    opts = cb.PlanOptions(mapping=mapping)
    y, name = planned(fft_transform(n, 2), x, opts)
    assert name == mapping, name
    ref, ref_name = planned(fft_transform(n, 2), x, cb.PlanOptions(mapping=mapping.split("[")[1].rstrip("]")))
    assert ref_name.startswith("fft-stockham-global"), ref_name
    assert _rel_l2_dev(y, ref) <= TOL, (name, ref_name)
    bins = np.sort(w.rng(80, log_n).integers(0, n, size=8))
    got = y[torch.as_tensor(bins + n, device=cuda)].cpu().numpy().view(np.complex64).reshape(-1)
    assert rel_l2(got, oracle.dft_bins(x[n:].cpu().numpy().view(np.complex64).reshape(-1), bins)) <= TOL
    back, _ = planned(fft_transform(n, 2, inverse=True, normalize=True), y, opts)
    assert _rel_l2_dev(back, x) <= TOL
    z = x.clone()
    z, zname = planned(fft_transform(n, 2, in_place=True), z)
    assert not zname.startswith("fft-l2-chain"), zname
    assert _rel_l2_dev(z, y) <= TOL


def test_fft_l2_chain_unaligned_workspace(lib, cuda):
    """The L2-chained plan drops its intermediate's lines from L2 once read;
    with a workspace that is 16-byte but not 128-byte aligned the
    intermediate still starts on a line of its own, so no line shared with
    other data is dropped: same result as the Stockham plan (rel L2 <= 2e-6)."""
    import torch

    n = 1 << 26
    x = w.torch_fft_input(n, 1, cuda, seed=5).reshape(n, 2)
    stream = torch.cuda.current_stream().cuda_stream
    with cb.Plan(lib, fft_transform(n, 1), options=cb.PlanOptions(mapping="fft-l2-chain[8+6+6+6]"),
                 stream=stream) as plan, \
            cb.Plan(lib, fft_transform(n, 1), options=cb.PlanOptions(mapping="8+6+6+6"), stream=stream) as ref:
        assert plan.algorithm_name() == "fft-l2-chain[8+6+6+6]"
        ws = torch.empty(plan.workspace_size() + 16, dtype=torch.uint8, device=cuda)
        plan.set_workspace(ws.data_ptr() + 16, plan.workspace_size())
        ref_ws = torch.empty(ref.workspace_size(), dtype=torch.uint8, device=cuda)
        ref.set_workspace(ref_ws.data_ptr(), ref.workspace_size())
        y, want = torch.empty_like(x), torch.empty_like(x)
        ref.execute(x.data_ptr(), want.data_ptr())
        for _ in range(2):
            y.zero_()
            plan.execute(x.data_ptr(), y.data_ptr())
            torch.cuda.synchronize()
            assert _rel_l2_dev(y, want) <= TOL
