"""Rank-two and rank-three R2C / C2R plans on the GPU through the C ABI.

R2C against the oracle's complex FFT of the real input along every axis (half
spectrum kept), C2R against the oracle's inverse of the Hermitian-completed
spectrum, and the round trip; relative L2 <= 2e-6."""
import math

import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def norm_scale(norm, inverse, volume):
    """numpy's normalisation modes as one output scale per direction."""
    return {"backward": (1.0, 1.0 / volume), "forward": (1.0 / volume, 1.0),
            "ortho": (1.0 / math.sqrt(volume),) * 2}[norm][int(inverse)]


def real_plan(lib, shape, batch, inverse, scale, cuda):
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.FP32, compute=cb.ComputeType.FP32, extents=list(shape),
                     batch=batch, inverse=inverse, normalize_inverse=False,
                     fft_type=cb.FftType.C2R if inverse else cb.FftType.R2C, fft_output_scale=scale,
                     execution_mode=cb.ExecutionMode.XD)
    plan = cb.Plan(lib, t, options=cb.PlanOptions(execution_mode=cb.ExecutionMode.XD),
                   stream=torch.cuda.current_stream().cuda_stream)
    ws = torch.empty(max(plan.workspace_size(), 16), dtype=torch.uint8, device=cuda)
    if plan.workspace_size():
        plan.set_workspace(ws.data_ptr(), plan.workspace_size())
    return plan, ws


def run_real(plan, x, out_shape, out_dtype, cuda):
    din = torch.from_numpy(np.ascontiguousarray(x)).to(cuda)
    dout = torch.empty(out_shape, dtype=out_dtype, device=cuda)
    plan.execute(din.data_ptr(), dout.data_ptr())
    torch.cuda.synchronize()
    return dout


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
    half_shape = (batch, *shape[:-1], h)
    fwd, ws_f = real_plan(lib, shape, batch, False, norm_scale(norm, False, vol), cuda)
    inv, ws_i = real_plan(lib, shape, batch, True, norm_scale(norm, True, vol), cuda)
    with fwd, inv:
        assert fwd.algorithm_name().startswith(f"fft-r2c-rank{len(shape)}[")
        spec = run_real(fwd, x, half_shape, torch.complex64, cuda)
        want = along_all_axes(oracle, x)[..., :h] * norm_scale(norm, False, vol)
        assert rel_l2(spec.cpu().numpy(), want) <= 2e-6
        # C2R of an exact half spectrum, and the round trip
        half = want.astype(np.complex64)
        back = run_real(inv, half, (batch, *shape), torch.float32, cuda)
        full = hermitian_full(half.astype(np.complex128), shape[-1])
        want_real = along_all_axes(oracle, full, inverse=True).real * norm_scale(norm, True, vol)
        assert rel_l2(back.cpu().numpy(), want_real) <= 2e-6
        again = run_real(inv, spec.cpu().numpy(), (batch, *shape), torch.float32, cuda)
        assert rel_l2(again.cpu().numpy(), x) <= 2e-6
