"""CPU-side contract of the PyTorch-facing operators: inputs that are not CUDA
tensors are rejected before any library call (no CPU fallback exists)."""
import pytest
import torch

from cubutterfly_b200 import torch_ops


def test_cpu_tensors_are_rejected():
    x = torch.randn(4, 64)
    for fn in (torch_ops.fwht, torch_ops.hadamard_rotate):
        with pytest.raises(ValueError, match="CUDA"):
            fn(x)
    with pytest.raises(ValueError, match="CUDA"):
        torch_ops.fft(x.to(torch.complex64))
    with pytest.raises(ValueError, match="CUDA"):
        torch_ops.zeta(torch.zeros(4, 64, dtype=torch.int32))
    with pytest.raises(ValueError, match="CUDA"):
        torch_ops.ntt(torch.zeros(4, 64, dtype=torch.int64), 998244353)


def test_inference_graph_needs_a_cuda_example():
    with pytest.raises(ValueError, match="CUDA Tensor example"):
        torch_ops.InferenceGraph(lambda v: v, torch.zeros(4))
