"""Short FP16 FWHT rows (N = 32, 64) with FP32 arithmetic and an explicit
caller scale applied before the single narrowing to FP16: the contract of the
reference's standalone provider python/cubutterfly/fused_short_fwht.py:15-80.

Here it is not a separately compiled module: the library's FWHT tile kernel
serves it through the C ABI (FP16 storage, FP32 compute, final-storage
rounding, output scale), one launch per call.  `prepare()` reports that
provider in the reference's metadata shape; `FusedShortFWHT` keeps its call
contract (CUDA FP16 tensor, contiguous last axis of 32 or 64, finite scale,
out of place).
"""
from __future__ import annotations

import hashlib
import math
from pathlib import Path

from . import default_library_path


def descriptor() -> dict:
    """Semantic contract of the provider (reference fused_short_fwht.py:29-50)."""
    return {
        "operator": "fwht",
        "storage_precision": "fp16",
        "accumulation": "fp32",
        "direction": "forward",
        "normalization": "caller-scale",
        "placement": "out-of-place",
        "layout": "contiguous-last-axis",
        "logN": [5, 6],
        "exchange": "warp-register",
        "launches": 1,
        "provider_kind": "linked-library-kernel",
        "requires_linked_provider": False,
        "fallback": None,
    }


def prepare(output=None, nvcc=None, sm=100) -> dict:
    """Metadata of the provider.  Nothing is compiled: the kernel is part of
    the library built by ``python -m cubutterfly_b200._build``; `output`,
    `nvcc` and `sm` are accepted for call compatibility and ignored."""
    del output, nvcc, sm
    module = Path(default_library_path()).resolve()
    return dict(provider="cubutterfly-b200-fwht-tile", public_search_integrated=True,
                candidate_descriptor=descriptor(), module=str(module),
                module_sha256=hashlib.sha256(module.read_bytes()).hexdigest() if module.is_file() else None,
                compile_command=None, supported_n=[32, 64], storage="fp16", accumulation="fp32",
                scale="explicit caller float; applied before single output narrowing", kernel_launches=1)


class FusedShortFWHT:
    """`FusedShortFWHT()(values, scale, out=None)`: H_N x * scale of every row
    of an FP16 CUDA tensor, N = 32 or 64.  `module` (a library path) is
    accepted for call compatibility; the in-tree library serves the call."""

    def __init__(self, module=None):
        self.module = Path(module).resolve() if module else Path(default_library_path()).resolve()

    def __call__(self, values, scale, out=None):
        import torch

        from . import torch_ops

        if not isinstance(values, torch.Tensor) or not values.is_cuda or values.dtype != torch.float16:
            raise ValueError("candidate requires a CUDA FP16 tensor")
        if values.ndim < 1 or values.shape[-1] not in (32, 64) or not values.is_contiguous():
            raise ValueError("candidate requires contiguous last-axis N32 or N64")
        if not math.isfinite(float(scale)) or not values.numel():
            raise ValueError("scale must be finite and batch nonempty")
        out = torch.empty_like(values) if out is None else out
        if (out.shape != values.shape or out.dtype != values.dtype or out.device != values.device
                or not out.is_contiguous()):
            raise ValueError("output must match contiguous input shape, dtype and device")
        if out.data_ptr() == values.data_ptr():
            raise ValueError("candidate is out-of-place")
        with torch.cuda.device(values.device):
            return torch_ops.fwht(values, scale=float(scale), out=out)
