"""Rank-two and rank-three R2C / C2R on the GPU: the C ABI plans and the
torch-facing RealFFT (the contract of the reference's
python/cubutterfly/real_fft.py).  R2C against the oracle's complex FFT of the
real input along every axis (half spectrum kept), C2R against the oracle's
inverse of the Hermitian-completed spectrum; relative L2 <= 2e-6."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w
from cubutterfly_b200.real_fft import RealFFT, output_scale

pytestmark = pytest.mark.gpu


def along_all_axes(oracle, x, inverse=False):
    """Unnormalised complex FFT of x (batch, *shape) along every axis but the batch."""
    y = x.astype(np.complex128)
    for axis in range(1, y.ndim):
        moved = np.moveaxis(y, axis, -1)
        shape = moved.shape
        out = oracle.fft_c64(np.ascontiguousarray(moved).reshape(-1, shape[-1]), inverse=inverse, normalize=False)
        y = np.moveaxis(out.reshape(shape), -1, axis)
    return y


def hermitian_full(half, n):
    """The full spectrum of a real signal from its half spectrum (last axis n)."""
    h = n // 2 + 1
    full = np.zeros(half.shape[:-1] + (n,), dtype=np.complex128)
    full[..., :h] = half
    mirror = np.conj(half[..., 1:n - h + 1][..., ::-1])  # bins n-1 .. h <- conj of bins 1 .. n-h
    for axis in range(1, half.ndim - 1):  # negate the outer frequency indices
        mirror = np.roll(np.flip(mirror, axis=axis), 1, axis=axis)
    full[..., h:] = mirror
    return full


@pytest.mark.parametrize("shape, batch", [((64, 128), 3), ((8, 16, 32), 2), ((256, 64), 1)])
@pytest.mark.parametrize("norm", ["backward", "ortho"])
def test_real_fft_rank_two_three(lib, oracle, cuda, shape, batch, norm):
    x = w.rng(90, sum(shape)).uniform(-1, 1, size=(batch, *shape)).astype(np.float32)
    vol = int(np.prod(shape))
    h = shape[-1] // 2 + 1
    with RealFFT(lib, shape, batch, cuda, norm=norm) as fft:
        assert fft.plans[0].algorithm_name().startswith(f"fft-r2c-rank{len(shape)}[")
        spec = fft.rfftn(torch.from_numpy(x).to(cuda))
        torch.cuda.synchronize()
        got = spec.cpu().numpy()
        want = along_all_axes(oracle, x)[..., :h] * output_scale(norm, False, vol)
        assert got.shape == (batch, *shape[:-1], h)
        assert rel_l2(got, want) <= 2e-6
        # C2R of an exact half spectrum, and the round trip
        half = want.astype(np.complex64)
        back = fft.irfftn(torch.from_numpy(half).to(cuda))
        torch.cuda.synchronize()
        full = hermitian_full(half.astype(np.complex128), shape[-1])
        want_real = along_all_axes(oracle, full, inverse=True).real * output_scale(norm, True, vol)
        assert rel_l2(back.cpu().numpy(), want_real) <= 2e-6
        assert rel_l2(fft.irfftn(spec).cpu().numpy(), x) <= 2e-6
        meta = fft.plan_metadata()
        assert [m["direction"] for m in meta] == ["forward", "inverse"]


def test_real_fft_contract_errors(lib, cuda):
    with pytest.raises(ValueError):
        RealFFT(lib, (64,), 1, cuda)
    with pytest.raises(ValueError):
        RealFFT(lib, (8, 8), 1, cuda, norm="none")
    with RealFFT(lib, (8, 16), 2, cuda, reuse_buffers=True) as fft:
        x = torch.zeros((2, 8, 16), dtype=torch.float32, device=cuda)
        a = fft.rfftn(x)
        assert fft.rfftn(x).data_ptr() == a.data_ptr()
        with pytest.raises(ValueError):
            fft.rfftn(torch.zeros((2, 8, 8), dtype=torch.float32, device=cuda))
        with pytest.raises(ValueError):
            fft.irfftn(x)  # real input to the C2R side
