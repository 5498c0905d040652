"""Prepared word64 RNS NTT plans over caller-owned CUDA buffers.

Public names are the reference's (python/cubutterfly/rns.py: ``Library``,
``Plan``, ``Placement``, ``CachePolicy``, ``Error``); the entry points are the
cubutterflyRns* C ABI of libcubutterfly_b200.so (include/cuntt/rns_c_api.h).

A plan moves through three states: created (config validated by the C side,
tables built), prepared (placement and mapping fixed, timed once unless a
cache answers), closed.  ``prepare`` runs once, outside stream capture and
timing; ``execute`` only enqueues the tile passes (no copies, no
synchronisation).  Buffers and streams must outlive the work enqueued on
them.  Importing this module loads nothing.
"""
from __future__ import annotations

import ctypes as ct
import json
import os
from enum import Enum, IntEnum

from . import _abi, default_library_path


class Error(RuntimeError):
    """A failed RNS call; `status` is 1 (invalid request) or 2 (runtime failure), None for frontend errors."""

    def __init__(self, message, status=None):
        super().__init__(message)
        self.status = status


class Placement(IntEnum):
    SEPARATE = 0
    IN_PLACE = 1


class CachePolicy(IntEnum):
    PREFER = 0
    REQUIRE = 1
    REFRESH = 2


_RNS_ABI = """
Create     s P
Prepare    p i s i w p
Execute    p p p p
InfoJson   p p Z
Destroy    p
LastError
"""


class Library:
    """The cubutterflyRns* entry points of a loaded libcubutterfly_b200.so."""

    def __init__(self, path=None):
        path = path if path is not None else default_library_path()
        if not os.path.isfile(path):
            raise FileNotFoundError(f"no cuButterfly library at {path}; build it with "
                                    "`python -m cubutterfly_b200._build`")
        self._dll = ct.CDLL(os.fspath(path))
        self.fn = _abi.bind(self._dll, "cubutterflyRns", _RNS_ABI, text=("LastError",))

    def invoke(self, name, *args):
        status = self.fn[name](*args)
        if status:
            detail = (self.fn["LastError"]() or b"").decode("utf-8", "replace")
            raise Error(detail or f"cubutterflyRns{name} failed with status {status}", status)

    def info_json(self, handle) -> dict:
        return json.loads(_abi.two_call_text(lambda *a: self.invoke("InfoJson", *a), handle))


def _payload(config) -> bytes:
    """The request as compact JSON text (the C parser validates every key)."""
    doc = json.loads(config) if isinstance(config, (str, bytes)) else config
    if not isinstance(doc, dict):
        raise TypeError(f"an RNS config is a JSON object (dict or text), not {type(doc).__name__}")
    return json.dumps(doc, allow_nan=False, separators=(",", ":")).encode("utf-8")


class _State(Enum):
    CREATED = "created"
    PREPARED = "prepared"
    CLOSED = "closed"


class Plan:
    """An owned RNS plan.  prepare() once, then execute(); close() releases it
    (explicitly, or by leaving a `with` block: nothing is freed from a
    finaliser while GPU work may still reference the plan)."""

    def __init__(self, library, config):
        self.library = library
        self._handle = ct.c_void_p()
        self._state = _State.CREATED
        self._placement = None
        library.invoke("Create", _payload(config), ct.byref(self._handle))
        if not self._handle.value:
            self._state = _State.CLOSED
            raise Error("cubutterflyRnsCreate reported success without a plan")

    def _need(self, *states):
        if self._state not in states:
            wanted = " or ".join(s.value for s in states)
            raise Error(f"RNS plan is {self._state.value}; this call needs a {wanted} plan")

    @property
    def native_handle(self):
        self._need(_State.CREATED, _State.PREPARED)
        return self._handle

    def prepare(self, *, placement=Placement.SEPARATE, cache_directory=None, policy=CachePolicy.PREFER,
                repetitions=5, stream=0):
        """Fix the placement and the mapping (timed `repetitions` times unless
        the cache in `cache_directory` answers, per `policy`).  Once per plan."""
        self._need(_State.CREATED)
        placement = Placement(_abi.unsigned(placement, "placement", ct.c_int))
        policy = CachePolicy(_abi.unsigned(policy, "policy", ct.c_int))
        reps = _abi.unsigned(repetitions, "repetitions", ct.c_uint)
        if reps < 1:
            raise ValueError("repetitions: at least one timed repetition is needed")
        where = os.fsencode(cache_directory) if cache_directory is not None else b""
        if b"\0" in where:
            raise ValueError("cache_directory: embedded NUL byte")
        self.library.invoke("Prepare", self._handle, int(placement), where, int(policy), reps,
                            _abi.address(stream, "stream"))
        self._placement = placement
        self._state = _State.PREPARED
        return self

    def execute(self, input, output, *, stream=0):
        """Enqueue the transform of `input` into `output` (device addresses, 8-byte aligned)."""
        self._need(_State.PREPARED)
        src = _abi.address(input, "input", nullable=False, align=8)
        dst = _abi.address(output, "output", nullable=False, align=8)
        aliased = src.value == dst.value
        if aliased != (self._placement is Placement.IN_PLACE):
            raise ValueError(f"the plan was prepared {self._placement.name.lower()}: input and output must "
                             + ("be the same buffer" if self._placement is Placement.IN_PLACE else "differ"))
        self.library.invoke("Execute", self._handle, src, dst, _abi.address(stream, "stream"))

    def info(self) -> dict:
        return self.library.info_json(self.native_handle)

    def close(self):
        if self._state is not _State.CLOSED:
            handle, self._handle, self._state = self._handle, ct.c_void_p(), _State.CLOSED
            self.library.invoke("Destroy", handle)

    def __enter__(self):
        self._need(_State.CREATED, _State.PREPARED)
        return self

    def __exit__(self, *exc):
        self.close()
