"""PyTorch-facing operators over the C ABI, and whole-function CUDA graphs.

The consumer side of the hot path: QuaRot-style Hadamard rotations of
activations (bf16/fp16/fp32 rows, FP32 arithmetic, one rounding at the end),
complex FFTs, zeta transforms and cyclic NTTs on torch tensors, launched on the
caller's current CUDA stream through plans that are built once per
(operator, shape, dtype, scale, orders, device, stream) and then reused.
Execution allocates nothing (workspaces are created with the plan), so the
calls are CUDA-graph capturable; ``InferenceGraph`` captures a whole
Tensor -> Tensor function with the contract of the reference's
``python/cubutterfly/torch_graph.py`` (InferenceGraph, :4-78).

torch is imported lazily; the library has no CPU fallback and raises when its
CUDA build is missing.
"""
from __future__ import annotations

import math
import threading

import cubutterfly_b200 as cb

__all__ = ["fwht", "hadamard_rotate", "fft", "zeta", "ntt", "plan_cache_size", "clear_plan_cache",
           "InferenceGraph"]

_LOCK = threading.Lock()
_PLANS: dict = {}


class _CachedPlan:
    """A plan bound to one stream, with its workspace held for its lifetime."""

    def __init__(self, transform, device, stream):
        import torch

        self.plan = cb.Plan(cb.load(), transform, stream=stream)
        self.workspace = None
        size = self.plan.workspace_size()
        if size:
            self.workspace = torch.empty(size, dtype=torch.uint8, device=device)
            self.plan.set_workspace(self.workspace.data_ptr(), size)


def _plan(key, transform, device, stream):
    with _LOCK:
        entry = _PLANS.get(key)
        if entry is None:
            import torch

            with torch.cuda.device(device):
                entry = _CachedPlan(transform, device, stream)
            _PLANS[key] = entry
        return entry.plan


def plan_cache_size() -> int:
    return len(_PLANS)


def clear_plan_cache() -> None:
    with _LOCK:
        for entry in _PLANS.values():
            entry.plan.close()
        _PLANS.clear()


def _check(x, dtypes, what):
    import torch

    if not isinstance(x, torch.Tensor) or not x.is_cuda:
        raise ValueError(f"{what} requires a CUDA tensor")
    if x.dtype not in dtypes:
        raise ValueError(f"{what} does not support dtype {x.dtype}")
    if x.ndim < 1 or x.numel() == 0:
        raise ValueError(f"{what} requires a non-empty tensor")
    n = x.shape[-1]
    if n < 2 or n & (n - 1):
        raise ValueError(f"{what} requires a power-of-two last dimension of at least 2")
    return n, x.numel() // n


def _run(key, transform, x, out):
    import torch

    stream = torch.cuda.current_stream(x.device)
    plan = _plan(key + (x.device.index, int(stream.cuda_stream)), transform, x.device, stream.cuda_stream)
    src = x.contiguous()
    if out is None:
        out = torch.empty_like(src)
    elif out.shape != src.shape or out.dtype != src.dtype or out.device != src.device or not out.is_contiguous():
        raise ValueError("out must be a contiguous tensor of the input's shape, dtype and device")
    if out.data_ptr() == src.data_ptr():
        raise ValueError("these operators are out of place: out must not alias the input")
    plan.execute(src.data_ptr(), out.data_ptr())
    return out


def _orders(transform, input_order, output_order):
    transform.input_orders = [int(input_order)]
    transform.output_orders = [int(output_order)]
    return transform


def fwht(x, scale: float = 1.0, inverse: bool = False, out=None,
         input_order=cb.LogicalOrder.NATURAL, output_order=cb.LogicalOrder.NATURAL):
    """Walsh-Hadamard transform of the last axis times `scale` (natural
    Hadamard order).  bf16 / fp16 tensors are widened to FP32, transformed and
    rounded once (final-storage rounding); fp32 tensors stay fp32.  An inverse
    transform is additionally scaled by 1/N."""
    import torch

    n, batch = _check(x, (torch.bfloat16, torch.float16, torch.float32), "fwht")
    if not math.isfinite(scale):
        raise ValueError("scale must be finite")
    storage = {torch.bfloat16: cb.DataType.BF16, torch.float16: cb.DataType.FP16,
               torch.float32: cb.DataType.FP32}[x.dtype]
    low = x.dtype != torch.float32
    t = cb.Transform(op=cb.Operator.FWHT, storage=storage, compute=cb.ComputeType.FP32, extents=[n], batch=batch,
                     inverse=inverse, output_scale=float(scale),
                     output_rounding=cb.OutputRounding.FINAL_STORAGE if low else cb.OutputRounding.STAGE_STORAGE)
    _orders(t, input_order, output_order)
    key = ("fwht", x.dtype, n, batch, bool(inverse), float(scale), int(input_order), int(output_order))
    return _run(key, t, x, out)


def hadamard_rotate(x, out=None):
    """The orthonormal rotation x -> x H_N / sqrt(N) of QuaRot-style quantisation
    (H_N symmetric, so this is also its own inverse)."""
    return fwht(x, scale=1.0 / math.sqrt(x.shape[-1]), out=out)


def fft(x, inverse: bool = False, normalize: bool = True, out=None,
        input_order=cb.LogicalOrder.NATURAL, output_order=cb.LogicalOrder.NATURAL):
    """Complex FFT of the last axis of a complex64 tensor (exp(-2 pi i jk/N)
    forward; the inverse is scaled by 1/N when `normalize`)."""
    import torch

    n, batch = _check(x, (torch.complex64,), "fft")
    t = cb.Transform(op=cb.Operator.FFT, storage=cb.DataType.COMPLEX_FP32, extents=[n], batch=batch,
                     inverse=inverse, normalize_inverse=normalize)
    _orders(t, input_order, output_order)
    key = ("fft", n, batch, bool(inverse), bool(normalize), int(input_order), int(output_order))
    return _run(key, t, x, out)


def zeta(x, superset: bool = False, inverse: bool = False, out=None):
    """Subset (or superset) zeta transform of the last axis, or its Moebius
    inverse, with wrap-around integer arithmetic.  int32 / int64 tensors carry
    uint32 / uint64 words."""
    import torch

    n, batch = _check(x, (torch.int32, torch.int64), "zeta")
    t = cb.Transform(op=cb.Operator.SUPERSET_ZETA if superset else cb.Operator.SUBSET_ZETA,
                     storage=cb.DataType.UINT32 if x.dtype == torch.int32 else cb.DataType.UINT64,
                     extents=[n], batch=batch, inverse=inverse)
    key = ("zeta", x.dtype, n, batch, bool(superset), bool(inverse))
    return _run(key, t, x, out)


def ntt(x, modulus: int, inverse: bool = False, out=None,
        input_order=cb.LogicalOrder.NATURAL, output_order=cb.LogicalOrder.NATURAL):
    """Cyclic NTT modulo a prime `modulus` of the last axis (root
    find_primitive_power_of_two_root(log N, q); inverse scaled by N^-1).
    int64 tensors carry uint64 words, int32 tensors uint32 words (q < 2^32)."""
    import torch

    n, batch = _check(x, (torch.int32, torch.int64), "ntt")
    word32 = x.dtype == torch.int32
    t = cb.Transform(op=cb.Operator.NTT, storage=cb.DataType.UINT32 if word32 else cb.DataType.UINT64,
                     extents=[n], batch=batch, modulus=int(modulus), word_bits=32 if word32 else 64,
                     inverse=inverse)
    _orders(t, input_order, output_order)
    key = ("ntt", x.dtype, n, batch, int(modulus), bool(inverse), int(input_order), int(output_order))
    return _run(key, t, x, out)


class InferenceGraph:
    """Capture a Tensor -> Tensor inference function for one fixed input contract.

    Construction warms the function up on `stream` and captures it in a CUDA
    graph.  Calls must be serialised on `stream` and use the captured shape,
    dtype and device; the callable (and any parameters) must stay alive and
    unchanged, and modules must be in eval mode.  Each call copies its input
    into the captured buffer, replays the graph and returns a clone of the
    output (independent storage, asynchronous on `stream`).  Autograd is not
    supported.  Same contract as the reference's torch_graph.InferenceGraph.
    """

    def __init__(self, function, example, *, stream=None, warmup=3):
        import torch

        if not isinstance(example, torch.Tensor) or not example.is_cuda:
            raise ValueError("a CUDA Tensor example is required")
        if example.requires_grad:
            raise ValueError("inference input must not require gradients")
        if warmup < 1:
            raise ValueError("warmup must be positive")
        self.torch = torch
        self.function = function
        self.shape, self.dtype, self.device = tuple(example.shape), example.dtype, example.device
        self.stream = stream if stream is not None else torch.cuda.Stream(device=self.device)
        if torch.device(self.stream.device) != self.device:
            raise ValueError("capture stream device differs from input device")
        if int(self.stream.cuda_stream) == 0:
            raise ValueError("capture requires a non-default CUDA stream")
        self._check_modules()
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream), torch.inference_mode():
            self._input = example.clone()
            for _ in range(warmup):  # builds every plan before capture
                output = function(self._input)
            if not isinstance(output, torch.Tensor):
                raise ValueError("inference function must return one Tensor")
        self.stream.synchronize()
        self._graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(self.stream), torch.inference_mode():
            with torch.cuda.graph(self._graph, stream=self.stream):
                self._output = function(self._input)
        self.stream.synchronize()

    def _check_modules(self):
        modules = getattr(self.function, "modules", None)
        if modules is not None and any(m.training for m in modules()):
            raise ValueError("all captured modules must be in eval mode")

    def _validate(self, value):
        torch = self.torch
        if not isinstance(value, torch.Tensor):
            raise ValueError("input must be a Tensor")
        if tuple(value.shape) != self.shape or value.dtype != self.dtype or value.device != self.device:
            raise ValueError("input shape/dtype/device differs from capture")
        if value.requires_grad:
            raise ValueError("inference input must not require gradients")
        if int(torch.cuda.current_stream(self.device).cuda_stream) != int(self.stream.cuda_stream):
            raise ValueError("call must run on the declared capture stream")
        self._check_modules()

    def __call__(self, value):
        self._validate(value)
        with self.torch.inference_mode():
            self._input.copy_(value)
            self._graph.replay()
            return self._output.clone()

    def contract(self):
        return dict(shape=list(self.shape), dtype=str(self.dtype), device=str(self.device),
                    stream=int(self.stream.cuda_stream), inference_only=True, serialized_calls=True,
                    input_copy_included=True,
                    output_ownership="independent clone per call; clone included in timing")
