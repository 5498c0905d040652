"""Descriptor inspection on the CPU: ``python -m cubutterfly_b200 FILE [FILE ...]``.

For each descriptor JSON file (``-`` reads standard input) prints one JSON
object: whether the descriptor is valid (with the library's reason when it is
not), its normalised form, its static capabilities and, with ``--mappings K``,
the planner's K best mappings for the current device or the builtin B200
profile (``cubutterflyB200RankMappings``).  No GPU is needed.  The exit status
is the number of invalid descriptors (capped at 100).
"""
from __future__ import annotations

import argparse
import ctypes as ct
import json
import sys

from . import Descriptor, Error, Library


def inspect(library: Library, text: str, mappings: int = 0) -> dict:
    report = {"valid": False}
    try:
        descriptor = Descriptor.from_json(library, text)
    except (Error, ValueError) as e:
        report["error"] = str(e)
        return report
    with descriptor:
        try:
            descriptor.validate()
            report["valid"] = True
        except Error as e:
            report["error"] = str(e)
        report["descriptor"] = json.loads(descriptor.json())
        report["capabilities"] = json.loads(descriptor.capabilities_json())
        if mappings and report["valid"]:
            size = ct.c_size_t()
            library.invoke("B200RankMappings", descriptor.native_handle, None, None, ct.byref(size))
            buf = ct.create_string_buffer(size.value)
            library.invoke("B200RankMappings", descriptor.native_handle, None, buf, ct.byref(size))
            report["mappings"] = json.loads(buf.value.decode())[:mappings]
    return report


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m cubutterfly_b200", description=__doc__.split("\n\n")[0])
    ap.add_argument("files", nargs="+", help="descriptor JSON files ('-': standard input)")
    ap.add_argument("--mappings", type=int, default=0, metavar="K", help="also list the K best mappings")
    ap.add_argument("--library", help="shared library (default: $CUBUTTERFLY_LIBRARY or the in-tree build)")
    ap.add_argument("--indent", type=int, default=None, help="pretty-print with this indent")
    args = ap.parse_args(argv)
    library = Library(args.library)
    invalid = 0
    for name in args.files:
        text = sys.stdin.read() if name == "-" else open(name, encoding="utf-8").read()
        report = {"file": name, **inspect(library, text, args.mappings)}
        invalid += not report["valid"]
        print(json.dumps(report, indent=args.indent))
    return min(invalid, 100)


if __name__ == "__main__":
    raise SystemExit(main())
