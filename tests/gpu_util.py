"""Helpers that drive the C ABI with torch-owned device buffers (GPU tests)."""
from __future__ import annotations

import numpy as np
import torch

import cubutterfly_b200 as cb


def stream_ptr() -> int:
    return torch.cuda.current_stream().cuda_stream


def to_device(a: np.ndarray, device) -> torch.Tensor:
    """Copy a numpy array's bytes into a device tensor (dtype-agnostic)."""
    a = np.ascontiguousarray(a)
    t = torch.from_numpy(a.view(np.uint8).reshape(-1).copy())
    return t.to(device)


def from_device(t: torch.Tensor, dtype, shape) -> np.ndarray:
    return t.cpu().numpy().view(dtype).reshape(shape)


def run(lib: cb.Library, transform: cb.Transform, x: np.ndarray, device, options=None, workspace=True):
    """Execute one plan on x (host array) through the C ABI; return the host result."""
    with cb.Plan(lib, transform, options=options, stream=stream_ptr()) as plan:
        din = to_device(x, device)
        assert plan.input_size() == din.numel(), (plan.input_size(), din.numel())
        dout = din if transform.in_place else torch.empty(plan.output_size(), dtype=torch.uint8, device=device)
        ws = None
        if plan.workspace_size():
            ws = torch.empty(plan.workspace_size(), dtype=torch.uint8, device=device)
            plan.set_workspace(ws.data_ptr(), ws.numel())
        plan.execute(din.data_ptr(), dout.data_ptr())
        torch.cuda.synchronize()
        return from_device(dout, x.dtype, x.shape), plan.algorithm_name()
