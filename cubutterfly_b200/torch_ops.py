"""PyTorch-facing operators over the C ABI, and whole-function CUDA graphs.

The consumer side of the hot path: QuaRot-style Hadamard rotations of
activations (bf16/fp16/fp32 rows, FP32 arithmetic, one rounding at the end),
complex FFTs, zeta transforms and cyclic NTTs on torch tensors, launched on the
caller's current CUDA stream through plans that are built once per
(operator, shape, dtype, scale, orders, device, stream) and then reused.
Execution allocates nothing (workspaces are created with the plan), so the
calls are CUDA-graph capturable; ``InferenceGraph`` captures a whole
Tensor -> Tensor function (the consumer the reference serves with
``python/cubutterfly/torch_graph.py``, same constructor and call).

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
    """A Tensor -> Tensor inference function (for example a Hadamard rotation
    feeding a model head) replayed as one CUDA graph for one input contract.

    `InferenceGraph(function, example, *, stream=None, warmup=3)` fixes the
    contract (the shape, dtype and CUDA device of `example`) and a capture
    stream (a new side stream unless given; never the legacy default stream).
    The function runs `warmup` times there first, which builds and caches
    every cuButterfly plan it needs, so no plan is created under capture; then
    it is captured once.  A call, made on the capture stream with a tensor of
    the contract, stages the value into the graph's static input, replays the
    graph and returns the static output copied into `out` (or a new tensor):
    all of it asynchronous on that stream.  The function and its parameters
    must stay unchanged, torch modules in eval mode; there is no autograd.
    """

    def __init__(self, function, example, *, stream=None, warmup=3):
        import torch

        self._torch = torch
        if not (isinstance(example, torch.Tensor) and example.is_cuda):
            raise ValueError("InferenceGraph needs a CUDA Tensor example to fix its input contract")
        self._key = (tuple(example.shape), example.dtype, example.device)
        self._reject_grad(example)
        if int(warmup) < 1:
            raise ValueError("warmup: at least one eager run must precede the capture")
        self.function = function
        self.shape, self.dtype, self.device = self._key
        self.stream = torch.cuda.Stream(device=self.device) if stream is None else stream
        if torch.device(self.stream.device) != self.device:
            raise ValueError(f"capture stream is on {self.stream.device}, the example on {self.device}")
        if int(self.stream.cuda_stream) == 0:
            raise ValueError("the legacy default stream cannot be captured; give a side stream")
        self._require_eval()
        self.stream.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(self.stream), torch.inference_mode():
            self._static_in = example.detach().clone()
            results = [function(self._static_in) for _ in range(int(warmup))]
            if not isinstance(results[-1], torch.Tensor):
                raise ValueError(f"the function returned {type(results[-1]).__name__}, not one Tensor")
            del results
            self.stream.synchronize()
            self._graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(self._graph, stream=self.stream):
                self._static_out = function(self._static_in)
        self.stream.synchronize()

    def _reject_grad(self, value):
        if value.requires_grad:
            raise ValueError("InferenceGraph is inference only: the input requires grad")

    def _require_eval(self):
        modules = getattr(self.function, "modules", None)
        if callable(modules) and any(m.training for m in modules()):
            raise ValueError("put every module of the function in eval mode before capture")

    def __call__(self, value, out=None):
        torch = self._torch
        if not isinstance(value, torch.Tensor) or (tuple(value.shape), value.dtype, value.device) != self._key:
            got = (tuple(value.shape), value.dtype, value.device) if isinstance(value, torch.Tensor) else type(value)
            raise ValueError(f"input {got} does not match the captured contract {self._key}")
        self._reject_grad(value)
        if int(torch.cuda.current_stream(self.device).cuda_stream) != int(self.stream.cuda_stream):
            raise ValueError("call the graph on its capture stream (with torch.cuda.stream(graph.stream))")
        self._require_eval()
        with torch.inference_mode():
            self._static_in.copy_(value)
            self._graph.replay()
            if out is None:
                return self._static_out.clone()
            return out.copy_(self._static_out)

    def contract(self):
        """The captured contract and call semantics, as a dict."""
        return {"shape": list(self.shape), "dtype": str(self.dtype), "device": str(self.device),
                "stream": int(self.stream.cuda_stream), "inference_only": True, "serialized_calls": True,
                "input_copy_included": True, "output": "copied into `out` or a new tensor on every call"}
