"""ctypes plumbing shared by the frontends (`cubutterfly_b200`, `.rns`).

Each C ABI is described by one signature table: a line per entry point, the
symbol's suffix followed by one code per argument (see ``ARG``).  ``bind``
resolves every symbol of a table once, so a missing export fails at load time
instead of at first use, and the bound callables are what the frontends call.
Arguments that cross the ABI go through ``unsigned`` / ``address`` first, which
reject bools, non-integers and values the C type cannot hold before any C code
runs.
"""
from __future__ import annotations

import ctypes as ct
import operator

# argument codes of the signature tables
ARG = {
    "p": ct.c_void_p,                 # handle, device pointer or opaque buffer
    "P": ct.POINTER(ct.c_void_p),     # handle out-parameter
    "i": ct.c_int,
    "I": ct.POINTER(ct.c_int),
    "u": ct.c_uint32,
    "U": ct.POINTER(ct.c_uint),
    "w": ct.c_uint,
    "q": ct.c_uint64,
    "z": ct.c_size_t,
    "Z": ct.POINTER(ct.c_size_t),
    "d": ct.c_double,
    "D": ct.POINTER(ct.c_double),
    "s": ct.c_char_p,
}


def parse_table(table: str) -> dict[str, list[str]]:
    """{suffix: [argument codes]} of a signature table (blank lines and # comments skipped)."""
    rows = {}
    for line in table.splitlines():
        line = line.split("#", 1)[0].split()
        if line:
            rows[line[0]] = line[1:]
    return rows


def bind(dll, prefix: str, table: str, *, text=(), extra=None) -> dict:
    """Resolve and type every entry point of `table` in `dll`.

    Entry points named in `text` return a C string; all others a status int.
    `extra` adds argument codes (e.g. a pointer to an ABI struct)."""
    codes = dict(ARG, **(extra or {}))
    bound = {}
    for suffix, args in parse_table(table).items():
        symbol = prefix + suffix
        try:
            fn = getattr(dll, symbol)
        except AttributeError:
            raise AttributeError(f"{symbol} is not exported by {dll._name}") from None
        fn.argtypes = [codes[a] for a in args]
        fn.restype = ct.c_char_p if suffix in text else ct.c_int
        bound[suffix] = fn
    return bound


_LIMITS = {ct.c_int: (0, (1 << 31) - 1)}


def unsigned(value, what: str, ctype=ct.c_size_t) -> int:
    """`value` as a non-negative Python int that `ctype` can hold."""
    if isinstance(value, bool):
        raise TypeError(f"{what}: a bool is not accepted where an integer is required")
    try:
        v = operator.index(value)
    except TypeError:
        raise TypeError(f"{what}: expected an integer, got {type(value).__name__}") from None
    lo, hi = _LIMITS.get(ctype, (0, (1 << (8 * ct.sizeof(ctype))) - 1))
    if not lo <= v <= hi:
        raise ValueError(f"{what}: {v} does not fit the ABI's {ctype.__name__} (0 .. {hi})")
    return v


def address(value, what: str = "pointer", *, nullable: bool = True, align: int = 1) -> ct.c_void_p:
    """A device or host address from an int, a c_void_p or anything with data_ptr() (torch tensors)."""
    if hasattr(value, "data_ptr"):
        value = value.data_ptr()
    elif isinstance(value, ct.c_void_p):
        value = value.value or 0
    elif value is None:
        value = 0
    v = unsigned(value, what, ct.c_void_p)
    if v == 0 and not nullable:
        raise ValueError(f"{what}: a null pointer is not accepted")
    if v % align:
        raise ValueError(f"{what}: address {v:#x} is not {align}-byte aligned")
    return ct.c_void_p(v)


def c_array(ctype, values):
    """A ctypes array of `values`, or NULL for an empty sequence."""
    values = list(values)
    return (ctype * len(values))(*values) if values else None


def two_call_text(fn, *head) -> str:
    """Run a two-call string query (size with a NULL buffer, then the text);
    `fn` is a checked call that raises when the ABI reports a failure."""
    size = ct.c_size_t(0)
    fn(*head, None, ct.byref(size))
    buf = ct.create_string_buffer(max(size.value, 1))
    fn(*head, buf, ct.byref(size))
    return buf.value.decode("utf-8")
