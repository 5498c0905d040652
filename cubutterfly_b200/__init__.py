"""Python frontend of libcubutterfly_b200.so (B200 planner + sm_100a kernels).

Public names, enum values and the call protocol are those of the reference's
Python package (python/cubutterfly/__init__.py: ``Library``, ``Transform``,
``PlanOptions``, ``Descriptor``, ``Plan``, ``Error`` and the enums), so code
written against it runs unchanged: ``Plan(Library(), Transform(...))`` then
``plan.execute(in_ptr, out_ptr)``.

How it is put together:

* ``_ABI`` is the one table of every C entry point this frontend binds (the
  reference ABI and the ``cubutterflyB200*`` extensions); ``Library`` binds it
  once at load time.
* A ``Transform`` (plus ``PlanOptions``) is first checked and normalised into a
  flat ``_Request`` by ``_request``; ``_SETTERS`` then lists, as data, the
  descriptor setters that configure it and the ``_Request`` fields each takes.

``Library()`` without a path loads ``$CUBUTTERFLY_LIBRARY`` or the in-tree
build and raises when neither exists: there is no CPU fallback.  Importing the
package loads nothing.  Execution is asynchronous; inputs, outputs, workspace
and stream must stay alive until it completes.
"""
from __future__ import annotations

import ctypes as ct
import json as _json
import os
from dataclasses import dataclass, field
from enum import IntEnum
from pathlib import Path
from types import SimpleNamespace

from . import _abi

__all__ = [
    "Operator", "DataType", "ComputeType", "LogicalOrder", "NttLayout", "ExecutionMode", "AlgorithmPolicy",
    "FftType", "LengthMode", "ArithmeticPolicy", "OutputRounding", "SelectionSource", "Status", "Transform",
    "PlanOptions", "Error", "Library", "Descriptor", "Plan", "default_library_path", "load",
]

_PKG = Path(__file__).resolve().parent
DEFAULT_LIBRARY = _PKG / "lib" / "libcubutterfly_b200.so"


def default_library_path() -> Path:
    """$CUBUTTERFLY_LIBRARY when set, else the in-tree build."""
    return Path(os.environ.get("CUBUTTERFLY_LIBRARY") or DEFAULT_LIBRARY)


# ---- enums: integer values fixed by include/cubutterfly/cubutterfly.h --------------------------
class Operator(IntEnum):
    FFT = 0
    NTT = 1
    FWHT = 2
    SUBSET_ZETA = 3
    SUPERSET_ZETA = 4
    STRUCTURED_2X2 = 5


class DataType(IntEnum):
    FP16 = 0
    BF16 = 1
    FP32 = 2
    FP64 = 3
    COMPLEX_FP16 = 4
    COMPLEX_BF16 = 5
    COMPLEX_FP32 = 6
    COMPLEX_FP64 = 7
    UINT32 = 8
    UINT64 = 9


class ComputeType(IntEnum):
    NATIVE = 0
    FP32 = 1
    FP64 = 2
    UINT32 = 3
    UINT64 = 4


class LogicalOrder(IntEnum):
    NATURAL = 0
    BIT_REVERSED = 1


class NttLayout(IntEnum):
    NATURAL = 0
    APPT_STATIC = 1
    BIT_REVERSED = 2


class ExecutionMode(IntEnum):
    AUTO = 0
    XD = 1
    COMPOSITE = 2


class AlgorithmPolicy(IntEnum):
    DEFAULT = 0
    MEASURE = 1
    EXPLICIT = 2


class FftType(IntEnum):
    C2C = 0
    R2C = 1
    C2R = 2


class LengthMode(IntEnum):
    STANDARD = 0
    ZERO_EXTENDED_EMBEDDING = 1


class ArithmeticPolicy(IntEnum):
    STRICT = 0
    ALLOW_FP16_MMA = 1


class OutputRounding(IntEnum):
    STAGE_STORAGE = 0
    FINAL_STORAGE = 1


class SelectionSource(IntEnum):
    MEASURED_TABLE = 0
    USER_CACHE = 1
    RUNTIME_MEASURED = 2
    STATIC_MODEL = 3
    EXPLICIT = 4
    UNMEASURED_FALLBACK = 5


class Status(IntEnum):
    SUCCESS = 0
    INVALID_VALUE = 1
    INVALID_TYPE = 2
    NOT_SUPPORTED = 3
    ALLOC_FAILED = 4
    CUDA_ERROR = 5
    BACKEND_ERROR = 6
    INTERNAL_ERROR = 7


DEFAULT_MODULUS = 1152921504606584833  # cuntt::kDefaultModulus


# ---- request records (field names and defaults are the reference's) ---------------------------
@dataclass
class Transform:
    """One batched transform request."""
    op: int = Operator.FFT
    storage: int = DataType.COMPLEX_FP32
    compute: int = ComputeType.NATIVE
    extents: list = field(default_factory=lambda: [256])
    batch: int = 1
    inverse: bool = False
    normalize_inverse: bool = True
    in_place: bool = False
    fft_type: int = FftType.C2C
    fft_output_scale: float = 1.0
    output_scale: float = 1.0
    output_rounding: int = OutputRounding.STAGE_STORAGE
    arithmetic_policy: int = ArithmeticPolicy.STRICT
    length_mode: int = LengthMode.STANDARD
    input_strides: list = field(default_factory=list)
    output_strides: list = field(default_factory=list)
    input_batch_stride: int = 0
    output_batch_stride: int = 0
    modulus: int = DEFAULT_MODULUS
    word_bits: int = 64
    stage_matrices: list = field(default_factory=list)
    input_orders: list = field(default_factory=list)
    output_orders: list = field(default_factory=list)
    input_order: int = NttLayout.NATURAL
    output_order: int = NttLayout.NATURAL
    execution_mode: int = ExecutionMode.AUTO


@dataclass
class PlanOptions:
    """Mapping selection: a policy, or an explicit mapping / algorithm name."""
    policy: int = AlgorithmPolicy.DEFAULT
    mapping: str = ""
    execution_mode: int = ExecutionMode.AUTO


class Error(RuntimeError):
    """A failed ABI call; `status` is the cubutterflyStatus_t value (None for frontend errors)."""

    def __init__(self, message, status=None):
        super().__init__(message)
        self.status = status


class _Matrix(ct.Structure):
    """cubutterflyMatrix2x2_t: [[m00, m01], [m10, m11]] applied to (left, right)."""
    _fields_ = [("m00", ct.c_double), ("m01", ct.c_double), ("m10", ct.c_double), ("m11", ct.c_double)]


# ---- the C ABI ---------------------------------------------------------------------------------
# suffix of cubutterfly<suffix>, then argument codes (_abi.ARG; "m": matrix array)
_ABI = """
GetStatusString            i
GetLastErrorString
GetVersion                 I I I
Create                     P
Destroy                    p
SetStream                  p p
GetStream                  p P
SetCachePath               p s
CreateDescriptor           P
DestroyDescriptor          p
SetOperator                p i
SetDataType                p i i
SetShape                   p u Z z
SetExecutionMode           p i
SetFftTransformType        p i
SetFftOutputScale          p d
SetOutputScale             p d
SetArithmeticPolicy        p i
SetOutputRounding          p i
SetStrides                 p Z z Z z
SetLogicalOrders           p I I
SetDirection               p i i
SetPlacement               p i
SetLengthMode              p i
SetAlgorithmPolicy         p i s
SetModulus                 p q u
SetNttLayouts              p i i
SetStageMatrices           p u m z
DescriptorValidate         p
DescriptorGetJson          p p Z
DescriptorSetJson          p s
DescriptorGetCapabilities  p p Z
CreatePlan                 p p P
DestroyPlan                p
PlanGetDescriptorJson      p p Z
PlanGetWorkspaceSize       p Z
PlanGetInputSize           p Z
PlanGetOutputSize          p Z
PlanGetPhysicalExtents     p Z u
PlanGetSelectionSource     p I
PlanGetAlgorithmName       p p Z
PlanGetSelectionReason     p p Z
PlanGetMappingJson         p p Z
PlanSetWorkspace           p p z
Execute                    p p p p
ExecuteSteady              p p p p
# extensions of this build (include/cubutterfly/cubutterfly_b200.h)
B200RankMappings           p s p Z
B200PlanGetDeviceStatus    p U
B200PlanInjectDeviceStatus p w
B200FourStepTwiddle        p z z z z z i p
B200PermuteBlocksC64       p p p p z z z z p
B200TransposeC64           p p z z z p
B200FftC2CNoAlloc          p p z z i i p
B200NttButterflyPeak       q D
B200PeerBufferCreate       z P p
B200PeerBufferOpen         p P
B200PeerBufferClose        p
B200PeerBufferDestroy      p
B200FourStepScatterColumns p p i i z z z z i p
B200FourStepScatterRows    p p i i z z z z i i p
B200FourStepScatterTranspose p p i i z z z z i p
"""


class Library:
    """libcubutterfly_b200.so with every entry point of `_ABI` bound."""

    def __init__(self, path=None):
        path = Path(path) if path else default_library_path()
        if not path.is_file():
            raise FileNotFoundError(
                f"no cuButterfly library at {path}; build it with `python -m cubutterfly_b200._build` "
                "(this frontend has no CPU fallback)")
        self.path = path
        self._dll = ct.CDLL(os.fspath(path))
        self.fn = _abi.bind(self._dll, "cubutterfly", _ABI, text=("GetStatusString", "GetLastErrorString"),
                            extra={"m": ct.POINTER(_Matrix)})

    def invoke(self, name, *args):
        """Call cubutterfly<name>; a nonzero status raises Error(status text: last error text)."""
        status = self.fn[name](*args)
        if status != Status.SUCCESS:
            raise Error(self.describe(status), status)

    def describe(self, status) -> str:
        text = (self.fn["GetStatusString"](int(status)) or b"").decode("utf-8", "replace")
        detail = (self.fn["GetLastErrorString"]() or b"").decode("utf-8", "replace")
        return f"{text}: {detail}" if detail else text

    def text(self, name, handle) -> str:
        """A two-call string query of `handle`."""
        return _abi.two_call_text(lambda *a: self.invoke(name, *a), handle)

    def version(self):
        v = [ct.c_int() for _ in range(3)]
        self.invoke("GetVersion", *(ct.byref(x) for x in v))
        return tuple(x.value for x in v)


_SHARED = {}


def load(path=None) -> Library:
    """A process-wide Library of `path` (default: the in-tree build)."""
    key = os.fspath(path) if path is not None else None
    if key not in _SHARED:
        _SHARED[key] = Library(path)
    return _SHARED[key]


# ---- Transform -> descriptor -----------------------------------------------------------------
_ENUM_FIELDS = ("op", "storage", "compute", "fft_type", "output_rounding", "arithmetic_policy", "length_mode",
                "input_order", "output_order", "execution_mode")
_SCALE_FIELDS = ("fft_output_scale", "output_scale")
_PER_AXIS = ("input_strides", "output_strides", "input_orders", "output_orders")


def _request(t: Transform, o: PlanOptions) -> SimpleNamespace:
    """Check a Transform + PlanOptions and flatten them into setter arguments."""
    r = SimpleNamespace()
    for flag in ("inverse", "normalize_inverse", "in_place"):
        if not isinstance(getattr(t, flag), bool):
            raise TypeError(f"Transform.{flag} takes True or False, got {getattr(t, flag)!r}")
    for name in _ENUM_FIELDS:
        setattr(r, name, _abi.unsigned(getattr(t, name), f"Transform.{name}", ct.c_int))
    for name in _SCALE_FIELDS:
        setattr(r, name, float(getattr(t, name)))
    for flag in ("inverse", "normalize_inverse", "in_place"):
        setattr(r, flag, getattr(t, flag))
    r.rank = _abi.unsigned(len(t.extents), "number of extents", ct.c_uint32)
    r.extents = [_abi.unsigned(e, "Transform.extents", ct.c_size_t) for e in t.extents]
    r.batch = _abi.unsigned(t.batch, "Transform.batch", ct.c_size_t)
    for name in _PER_AXIS:
        values = list(getattr(t, name))
        if values and len(values) != r.rank:
            raise ValueError(f"Transform.{name} has {len(values)} entries for {r.rank} axes (one per axis, or none)")
        kind = ct.c_size_t if name.endswith("strides") else ct.c_int
        setattr(r, name, [_abi.unsigned(v, f"Transform.{name}", kind) for v in values])
    r.input_batch_stride = _abi.unsigned(t.input_batch_stride, "Transform.input_batch_stride")
    r.output_batch_stride = _abi.unsigned(t.output_batch_stride, "Transform.output_batch_stride")
    r.modulus = _abi.unsigned(t.modulus, "Transform.modulus", ct.c_uint64)
    r.word_bits = _abi.unsigned(t.word_bits, "Transform.word_bits", ct.c_uint32)
    r.ntt = r.op == Operator.NTT
    # the legacy rank-one NTT layouts and per-axis logical orders are two ways
    # of saying the same thing: a request may use one of them
    r.legacy_layouts = (r.input_order, r.output_order) != (NttLayout.NATURAL, NttLayout.NATURAL)
    if r.legacy_layouts and not r.ntt:
        raise ValueError("input_order / output_order (NTT layouts) apply to NTT transforms only; "
                         "use input_orders / output_orders")
    if r.legacy_layouts and (r.input_orders or r.output_orders):
        raise ValueError("give either NTT layouts (input_order / output_order) or logical orders "
                         "(input_orders / output_orders), not both")
    if not r.ntt and (r.modulus, r.word_bits) != (DEFAULT_MODULUS, 64):
        raise ValueError(f"modulus / word_bits are NTT parameters; {Operator(r.op).name if r.op in set(Operator) else r.op} "
                         "transforms take the defaults")
    r.matrices = []
    for axis, stages in enumerate(t.stage_matrices):
        _abi.unsigned(axis, "stage matrix axis", ct.c_uint32)
        if stages:
            r.matrices.append((axis, [_Matrix(*m) for m in stages]))
    r.policy = _abi.unsigned(o.policy, "PlanOptions.policy", ct.c_int)
    r.mapping = o.mapping.encode("utf-8")
    if r.mapping:
        r.policy = AlgorithmPolicy.EXPLICIT
    r.mode = _abi.unsigned(o.execution_mode, "PlanOptions.execution_mode", ct.c_int) or r.execution_mode
    return r


def _arr(kind, values):
    return _abi.c_array(kind, values)


# Descriptor setters in call order, each with a predicate (None: always) and
# the arguments it takes from a _Request.  SetShape clears strides, orders and
# stage matrices, so everything per-axis follows it.
_SETTERS = (
    ("SetOperator", None, lambda r: (r.op,)),
    ("SetShape", None, lambda r: (r.rank, _arr(ct.c_size_t, r.extents), r.batch)),
    ("SetDataType", None, lambda r: (r.storage, r.compute)),
    ("SetDirection", None, lambda r: (int(r.inverse), int(r.normalize_inverse))),
    ("SetPlacement", None, lambda r: (int(r.in_place),)),
    ("SetExecutionMode", None, lambda r: (r.mode,)),
    ("SetLengthMode", None, lambda r: (r.length_mode,)),
    ("SetFftTransformType", None, lambda r: (r.fft_type,)),
    ("SetFftOutputScale", None, lambda r: (r.fft_output_scale,)),
    ("SetOutputScale", None, lambda r: (r.output_scale,)),
    ("SetOutputRounding", None, lambda r: (r.output_rounding,)),
    ("SetArithmeticPolicy", None, lambda r: (r.arithmetic_policy,)),
    ("SetStrides", None, lambda r: (_arr(ct.c_size_t, r.input_strides), r.input_batch_stride,
                                    _arr(ct.c_size_t, r.output_strides), r.output_batch_stride)),
    ("SetModulus", lambda r: r.ntt, lambda r: (r.modulus, r.word_bits)),
    ("SetNttLayouts", lambda r: r.ntt, lambda r: (r.input_order, r.output_order)),
    ("SetLogicalOrders", lambda r: not r.legacy_layouts,
     lambda r: (_arr(ct.c_int, r.input_orders), _arr(ct.c_int, r.output_orders))),
    ("SetAlgorithmPolicy", None, lambda r: (r.policy, r.mapping)),
)


class Descriptor:
    """An owned cubutterflyDescriptor_t, configured from a Transform or loaded from JSON."""

    def __init__(self, library, transform, options=None):
        self.library = library
        self._handle = ct.c_void_p()
        library.invoke("CreateDescriptor", ct.byref(self._handle))
        try:
            self._apply(_request(transform, options or PlanOptions()))
        except BaseException:
            self.close()
            raise

    def _apply(self, r):
        for name, when, args in _SETTERS:
            if when is None or when(r):
                self.library.invoke(name, self._handle, *args(r))
        for axis, stages in r.matrices:
            self.library.invoke("SetStageMatrices", self._handle, axis, _arr(_Matrix, stages), len(stages))

    @classmethod
    def from_json(cls, library, value):
        """A descriptor from its JSON document (a str, or a dict serialised here)."""
        self = cls.__new__(cls)
        self.library, self._handle = library, ct.c_void_p()
        library.invoke("CreateDescriptor", ct.byref(self._handle))
        try:
            text = value if isinstance(value, str) else _json.dumps(value)
            library.invoke("DescriptorSetJson", self._handle, text.encode("utf-8"))
        except BaseException:
            self.close()
            raise
        return self

    @property
    def native_handle(self):
        if not self._handle.value:
            raise Error("this Descriptor has been closed")
        return self._handle

    def validate(self):
        self.library.invoke("DescriptorValidate", self.native_handle)

    def json(self):
        return self.library.text("DescriptorGetJson", self.native_handle)

    def capabilities_json(self):
        return self.library.text("DescriptorGetCapabilities", self.native_handle)

    def close(self):
        handle, self._handle = self._handle, ct.c_void_p()
        if handle.value:
            self.library.invoke("DestroyDescriptor", handle)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


class Plan:
    """An immutable plan and the handle (stream context) it executes on.

    `transform` is a Transform (with optional PlanOptions) or a Descriptor of
    the same Library.  The stream is fixed at construction.  Workspace is the
    caller's: query workspace_size(), allocate, bind with set_workspace(),
    which also keeps the passed object alive.  execute() is asynchronous;
    pointers may be ints, c_void_p or objects with data_ptr() (torch tensors).
    """

    def __init__(self, library, transform, options=None, stream=None, cache_path=None):
        self.library = library
        self._context, self._handle = ct.c_void_p(), ct.c_void_p()
        self._workspace = None
        try:
            library.invoke("Create", ct.byref(self._context))
            cache = os.environ.get("CUBUTTERFLY_PLAN_CACHE") if cache_path is None else cache_path
            if cache:
                library.invoke("SetCachePath", self._context, os.fsencode(cache))
            if stream is not None:
                library.invoke("SetStream", self._context, _abi.address(stream, "stream"))
            if isinstance(transform, Descriptor):
                if options is not None:
                    raise ValueError("a Descriptor carries its own selection; pass options when building it")
                if transform.library is not library:
                    raise ValueError("the Descriptor was created by a different Library")
                self._create(transform)
            else:
                with Descriptor(library, transform, options) as d:
                    self._create(d)
        except BaseException:
            self.close()
            raise

    def _create(self, descriptor):
        self.library.invoke("CreatePlan", self._context, descriptor.native_handle, ct.byref(self._handle))

    @property
    def native_handle(self):
        if not self._handle.value:
            raise Error("this Plan has been closed")
        return self._handle

    @property
    def native_context(self):
        if not self._context.value:
            raise Error("this Plan has been closed")
        return self._context

    def set_stream(self, stream):
        raise Error("a plan's stream is fixed when it is created: pass stream= to Plan()")

    def _bytes(self, query):
        v = ct.c_size_t()
        self.library.invoke(query, self.native_handle, ct.byref(v))
        return v.value

    def workspace_size(self):
        return self._bytes("PlanGetWorkspaceSize")

    def input_size(self):
        return self._bytes("PlanGetInputSize")

    def output_size(self):
        return self._bytes("PlanGetOutputSize")

    def selection_source(self):
        v = ct.c_int()
        self.library.invoke("PlanGetSelectionSource", self.native_handle, ct.byref(v))
        return SelectionSource(v.value)

    def set_workspace(self, pointer, bytes):
        self.library.invoke("PlanSetWorkspace", self.native_handle, _abi.address(pointer, "workspace"),
                            _abi.unsigned(bytes, "workspace bytes"))
        self._workspace = pointer

    def physical_extents(self, rank):
        """Extents the plan transforms physically: the padded length of a
        zero-extended embedding, the convolution length of a non-power-of-two
        FFT axis, else the logical extent."""
        out = (ct.c_size_t * rank)()
        self.library.invoke("PlanGetPhysicalExtents", self.native_handle, out, rank)
        return list(out)

    def execute(self, input, output):
        self.library.invoke("Execute", self.native_context, self.native_handle, _abi.address(input, "input"),
                            _abi.address(output, "output"))

    def execute_steady(self, input, output):
        self.library.invoke("ExecuteSteady", self.native_context, self.native_handle, _abi.address(input, "input"),
                            _abi.address(output, "output"))

    def device_status(self) -> int:
        """Failure bits recorded on the device by earlier launches (0: none);
        final once the plan's stream has been synchronised."""
        v = ct.c_uint()
        self.library.invoke("B200PlanGetDeviceStatus", self.native_handle, ct.byref(v))
        return v.value

    def inject_device_status(self, bits: int):
        """Test hook: record `bits` as a failing launch would."""
        self.library.invoke("B200PlanInjectDeviceStatus", self.native_handle, _abi.unsigned(bits, "bits", ct.c_uint))

    def mapping_json(self):
        return self.library.text("PlanGetMappingJson", self.native_handle)

    def descriptor_json(self):
        return self.library.text("PlanGetDescriptorJson", self.native_handle)

    def algorithm_name(self):
        return self.library.text("PlanGetAlgorithmName", self.native_handle)

    def selection_reason(self):
        return self.library.text("PlanGetSelectionReason", self.native_handle)

    def close(self):
        handle, self._handle = self._handle, ct.c_void_p()
        context, self._context = self._context, ct.c_void_p()
        self._workspace = None
        try:
            if handle.value:
                self.library.invoke("DestroyPlan", handle)
        finally:
            if context.value:
                self.library.invoke("Destroy", context)

    def __enter__(self):
        return self

    def __exit__(self, *exc):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
