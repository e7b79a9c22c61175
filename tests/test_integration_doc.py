"""The Zig binding a maintainer adds (`src/dnb.zig`) declares every entry point of
include/dnb200.h with the same number of arguments, so the drop-in list cannot fall behind the
header."""
from __future__ import annotations

import os
import re

from darknet_zig_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _zig_externs() -> dict[str, int]:
    text = open(os.path.join(ROOT, "INTEGRATION.md")).read()
    out = {}
    for m in re.finditer(r"pub extern fn (dnb_\w+)\(([^)]*)\)", text):
        args = [a for a in m.group(2).split(",") if a.strip()]
        out[m.group(1)] = len(args)
    return out


def _header_arity() -> dict[str, int]:
    text = open(os.path.join(ROOT, "include", "dnb200.h")).read()
    text = re.sub(r"/\*.*?\*/", " ", text, flags=re.S)
    out = {}
    for m in re.finditer(r"\b(dnb_\w+)\s*\(([^;{]*?)\)\s*;", text):
        args = m.group(2).strip()
        out[m.group(1)] = 0 if args in ("", "void") else len(args.split(","))
    return out


def test_every_entry_point_has_a_zig_extern():
    declared = set(_lib.declared_symbols())
    zig = _zig_externs()
    assert declared - set(zig) == set(), f"missing from INTEGRATION.md: {sorted(declared - set(zig))}"
    assert set(zig) - declared == set(), f"not in the header: {sorted(set(zig) - declared)}"


def test_zig_externs_take_the_header_arguments():
    header = _header_arity()
    for name, n in _zig_externs().items():
        assert header.get(name) == n, f"{name}: {n} arguments in INTEGRATION.md, {header.get(name)} in the header"
