"""Prepared word64 RNS NTT plans over caller-owned CUDA buffers.

Mirrors the reference's python/cubutterfly/rns.py:67-170 (Library, Plan,
Placement, CachePolicy, Error; prepare -> execute -> info -> close) over the
cubutterflyRns* C ABI of libcubutterfly_b200.so.  Import loads nothing.
Prepare belongs outside stream capture and timing; execute enqueues the two
tile passes without copying or synchronising.
"""
from __future__ import annotations

import ctypes as ct
import json
import operator
import os
from enum import IntEnum
from pathlib import Path

from . import default_library_path


class Error(RuntimeError):
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


def _integer(value, name, maximum):
    if isinstance(value, bool):
        raise TypeError(f"{name} must be an integer, not bool")
    try:
        value = operator.index(value)
    except TypeError as exc:
        raise TypeError(f"{name} must be an integer") from exc
    if not 0 <= value <= maximum:
        raise ValueError(f"{name} is outside the ABI range")
    return value


def _pointer(value, name, *, nullable=False, aligned=False):
    if hasattr(value, "data_ptr"):
        value = value.data_ptr()
    if isinstance(value, ct.c_void_p):
        value = value.value or 0
    value = _integer(value, name, (1 << (ct.sizeof(ct.c_void_p) * 8)) - 1)
    if not nullable and not value:
        raise ValueError(f"{name} must be non-null")
    if aligned and value % ct.alignment(ct.c_uint64):
        raise ValueError(f"{name} must be uint64 aligned")
    return ct.c_void_p(value)


def _config_json(config):
    if isinstance(config, str):
        config = json.loads(config)
    if not isinstance(config, dict):
        raise TypeError("config must be a dict or JSON object string")
    return json.dumps(config, allow_nan=False, separators=(",", ":")).encode("utf-8")


class Library:
    """The RNS entry points of a loaded libcubutterfly_b200.so."""

    def __init__(self, path=None):
        path = Path(path) if path else default_library_path()
        if not path.exists():
            raise FileNotFoundError(f"{path} is missing: build it with `python -m cubutterfly_b200._build`")
        self._dll = ct.CDLL(os.fspath(path))
        p = ct.c_void_p
        sig = {
            "Create": [ct.c_char_p, ct.POINTER(p)],
            "Prepare": [p, ct.c_int, ct.c_char_p, ct.c_int, ct.c_uint, p],
            "Execute": [p, p, p, p],
            "InfoJson": [p, p, ct.POINTER(ct.c_size_t)],
            "Destroy": [p],
            "LastError": [],
        }
        for name, args in sig.items():
            fn = getattr(self._dll, "cubutterflyRns" + name)
            fn.argtypes = args
            fn.restype = ct.c_char_p if name == "LastError" else ct.c_int

    def _call(self, name, *args):
        status = getattr(self._dll, "cubutterflyRns" + name)(*args)
        if status:
            message = self._dll.cubutterflyRnsLastError() or b"RNS operation failed"
            raise Error(message.decode("utf-8", errors="replace"), status)

    def _info(self, handle):
        size = ct.c_size_t()
        self._call("InfoJson", handle, None, ct.byref(size))
        buf = ct.create_string_buffer(size.value)
        self._call("InfoJson", handle, buf, ct.byref(size))
        return json.loads(buf.value.decode("utf-8"))


class Plan:
    """Owned RNS plan.  prepare() must succeed before execute(); close() explicitly."""

    def __init__(self, library, config):
        self.library = library
        self._handle = ct.c_void_p()
        self._placement = None
        library._call("Create", _config_json(config), ct.byref(self._handle))
        if not self._handle.value:
            raise Error("RNS Create returned a null plan")

    @property
    def native_handle(self):
        if not self._handle.value:
            raise Error("RNS plan is closed")
        return self._handle

    def prepare(self, *, placement=Placement.SEPARATE, cache_directory=None, policy=CachePolicy.PREFER,
                repetitions=5, stream=0):
        handle = self.native_handle
        if self._placement is not None:
            raise Error("plan is already prepared; create another plan to retune")
        placement = Placement(_integer(placement, "placement", 1))
        policy = CachePolicy(_integer(policy, "policy", 2))
        repetitions = _integer(repetitions, "repetitions", (1 << 32) - 1)
        if not repetitions:
            raise ValueError("repetitions must be positive")
        directory = b"" if cache_directory is None else os.fsencode(cache_directory)
        if b"\0" in directory:
            raise ValueError("cache_directory must not contain NUL")
        self.library._call("Prepare", handle, int(placement), directory, int(policy), repetitions,
                           _pointer(stream, "stream", nullable=True))
        self._placement = placement
        return self

    def execute(self, input, output, *, stream=0):
        handle = self.native_handle
        if self._placement is None:
            raise Error("RNS plan must be prepared before execution")
        src = _pointer(input, "input", aligned=True)
        dst = _pointer(output, "output", aligned=True)
        if (src.value == dst.value) != (self._placement == Placement.IN_PLACE):
            raise ValueError("pointer aliasing does not match prepared placement")
        self.library._call("Execute", handle, src, dst, _pointer(stream, "stream", nullable=True))

    def info(self):
        return self.library._info(self.native_handle)

    def close(self):
        if self._handle.value:
            self.library._call("Destroy", self._handle)
            self._handle = ct.c_void_p()

    def __enter__(self):
        self.native_handle
        return self

    def __exit__(self, *exc):
        self.close()
