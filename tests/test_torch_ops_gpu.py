"""PyTorch-facing operators and whole-function CUDA graphs on the GPU: the
QuaRot-style Hadamard rotation, FFT, zeta and NTT on torch tensors against the
oracle, plan reuse, and InferenceGraph capture/replay of a rotation."""
import numpy as np
import pytest
import torch

import cubutterfly_b200 as cb
from conftest import rel_l2
from cubutterfly_b200 import torch_ops
from cubutterfly_b200 import workloads as w

pytestmark = pytest.mark.gpu


def test_hadamard_rotation_bf16_matches_oracle(oracle, cuda):
    bits = w.fwht_input_bits(64, 4096, seed=5)
    x = torch.from_numpy(bits.view(np.int16).copy()).view(torch.bfloat16).to(cuda)
    y = torch_ops.hadamard_rotate(x)
    got = y.view(torch.int16).cpu().numpy().view(np.uint16)
    want = oracle.fwht_bf16_final(bits, 1 / 64.0)
    assert rel_l2(w.bf16_bits_to_f32(got), w.bf16_bits_to_f32(want)) <= 4e-3
    assert np.mean(got == want) > 0.99


def test_rotation_is_orthonormal_in_fp32(cuda):
    x = torch.randn(32, 1024, device=cuda)
    y = torch_ops.hadamard_rotate(torch_ops.hadamard_rotate(x))
    assert torch.allclose(y, x, atol=1e-5)
    assert torch.allclose(torch_ops.hadamard_rotate(x).norm(dim=-1), x.norm(dim=-1), rtol=1e-5)


def test_fft_zeta_ntt_on_tensors(oracle, cuda):
    xf = w.fft_input(2048, 3, seed=2)
    got = torch_ops.fft(torch.from_numpy(xf).to(cuda)).cpu().numpy()
    assert rel_l2(got, oracle.fft_c32(xf)) <= 2e-6
    z = w.zeta_input(12, 2, seed=3)
    got = torch_ops.zeta(torch.from_numpy(z.view(np.int32)).to(cuda)).cpu().numpy().view(np.uint32)
    assert np.array_equal(got, oracle.zeta(z))
    q = 998244353
    v = w.rng(4).integers(0, q, size=(4, 1 << 13), dtype=np.uint64)
    got = torch_ops.ntt(torch.from_numpy(v.view(np.int64)).to(cuda), q).cpu().numpy().view(np.uint64)
    assert np.array_equal(got, oracle.ntt_cyclic(v, q))
    back = torch_ops.ntt(torch.from_numpy(got.view(np.int64)).to(cuda), q, inverse=True)
    assert np.array_equal(back.cpu().numpy().view(np.uint64), v)


def test_plans_are_reused_per_stream(cuda):
    torch_ops.clear_plan_cache()
    x = torch.randn(8, 256, device=cuda)
    for _ in range(3):
        torch_ops.fwht(x)
    assert torch_ops.plan_cache_size() == 1
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        torch_ops.fwht(x)
    s.synchronize()
    assert torch_ops.plan_cache_size() == 2


def test_inference_graph_replays_a_rotation(cuda):
    x = torch.randn(128, 4096, device=cuda).to(torch.bfloat16)

    def rotate_and_scale(v):
        return torch_ops.hadamard_rotate(v) * 2

    g = torch_ops.InferenceGraph(rotate_and_scale, x)
    with torch.cuda.stream(g.stream):
        for seed in range(3):
            v = torch.randn(128, 4096, device=cuda, generator=torch.Generator(cuda).manual_seed(seed))
            v = v.to(torch.bfloat16)
            got = g(v)
            want = rotate_and_scale(v)
            assert torch.equal(got, want)
    g.stream.synchronize()
    with pytest.raises(ValueError):
        g(x)  # not on the capture stream
    assert g.contract()["inference_only"]


def test_operators_reject_bad_tensors(cuda):
    with pytest.raises(ValueError):
        torch_ops.fwht(torch.randn(4, 100, device=cuda))  # not a power of two
    x = torch.randn(4, 64, device=cuda)
    with pytest.raises(ValueError):
        torch_ops.fwht(x, out=x)  # aliasing
    with pytest.raises(ValueError):
        torch_ops.fft(torch.randn(4, 64, device=cuda))  # not complex
