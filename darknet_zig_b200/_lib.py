"""Loads libdnb200.so and binds every entry point declared in include/dnb200.h.

The ctypes signatures are read from the header itself, so the header stays the single
description of the ABI. Loading fails loudly: there is no CPU fallback anywhere in this
package, and an op whose library is missing raises instead of computing something else.
"""
from __future__ import annotations

import ctypes as C
import os
import re
import threading

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
HEADER = os.path.join(ROOT, "include", "dnb200.h")
LIB_PATH = os.environ.get("DARKNET_KERNELS") or os.path.join(PKG, "libdnb200.so")

_CTYPES = {
    "int64_t": C.c_int64,
    "int": C.c_int,
    "float": C.c_float,
    "size_t": C.c_size_t,
    "dnb_stream": C.c_void_p,
    "dnb_comm": C.c_void_p,
    "dnb_dpsgd": C.c_void_p,
    "dnb_status": C.c_int,
}

_DECL = re.compile(r"^(dnb_status|const char \*)\s*(dnb_\w+)\((.*?)\);", re.S | re.M)


def parse_header(path: str = HEADER) -> dict[str, tuple[object, list[object]]]:
    """{name: (restype, [argtypes])} for every function declared in the header."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    out = {}
    for ret, name, args in _DECL.findall(text):
        restype = C.c_char_p if ret.startswith("const char") else C.c_int
        argtypes = []
        args = " ".join(args.split())
        if args and args != "void":
            for a in args.split(","):
                a = a.strip()
                if "*" in a:
                    argtypes.append(C.c_void_p)
                    continue
                typ = " ".join(a.replace("const ", "").split()[:-1])
                argtypes.append(_CTYPES[typ])
        out[name] = (restype, argtypes)
    return out


class DnbError(RuntimeError):
    """A libdnb200 call returned a non-zero dnb_status."""

    def __init__(self, status: int, what: str, detail: str):
        self.status = status
        super().__init__(f"{what}: {detail or 'status %d' % status}")


_lock = threading.Lock()
_lib = None
_sigs = None


def lib():
    """The loaded library with typed entry points (loaded once)."""
    global _lib, _sigs
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(
                    f"libdnb200.so not found at {LIB_PATH}; build it with `python -m darknet_zig_b200.build`")
            handle = C.CDLL(LIB_PATH)
            _sigs = parse_header()
            for name, (restype, argtypes) in _sigs.items():
                fn = getattr(handle, name)
                fn.restype = restype
                fn.argtypes = argtypes
            _lib = handle
    return _lib


def declared_symbols() -> list[str]:
    return sorted(parse_header().keys())


def call(name: str, *args) -> None:
    """Calls dnb_<name>(*args) and raises DnbError on a non-zero status. The argument count
    must match the header's: ctypes would convert surplus arguments by guesswork (a pointer
    passed as a C int is truncated) instead of refusing them."""
    L = lib()
    fn = getattr(L, "dnb_" + name)
    if len(args) != len(fn.argtypes):
        raise TypeError(f"dnb_{name} takes {len(fn.argtypes)} arguments, {len(args)} given")
    st = fn(*args)
    if st != 0:
        detail = L.dnb_last_error_detail()
        detail = detail.decode() if detail else ""
        err = L.dnb_error_string(st)
        raise DnbError(st, f"dnb_{name} failed ({err.decode() if err else st})", detail)
