"""The C ABI on the CPU: the library builds for sm_100a, loads, exports every entry point
include/dnb200.h declares, and rejects bad arguments before touching a device."""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import pytest

from darknet_zig_b200 import _lib


def test_library_exports_every_declared_symbol(built_lib):
    declared = _lib.declared_symbols()
    assert len(declared) >= 50
    out = subprocess.run(["nm", "-D", "--defined-only", built_lib], capture_output=True, text=True, check=True).stdout
    exported = {line.split()[-1] for line in out.splitlines() if " T " in line}
    missing = [s for s in declared if s not in exported]
    assert not missing, f"declared but not exported: {missing}"
    lib = _lib.lib()
    for s in declared:
        assert getattr(lib, s) is not None


def test_library_is_built_for_sm100a(built_lib):
    """The embedded device code is named for sm_100a (the file list only; the tool is the
    one next to the nvcc the build uses)."""
    from darknet_zig_b200 import build

    nvcc = build.nvcc_path()
    tool = os.path.join(os.path.dirname(nvcc), "cuobjdump") if nvcc else ""
    if not tool or not os.path.exists(tool):
        pytest.skip(f"no cuobjdump beside the nvcc the build uses ({nvcc})")
    out = subprocess.run([tool, "--list-elf", built_lib], capture_output=True, text=True)
    assert "sm_100a" in out.stdout


def test_error_strings(built_lib):
    lib = _lib.lib()
    for code in range(8):
        assert lib.dnb_error_string(code)
    assert lib.dnb_error_string(3) == b"device-side wait timed out"


@pytest.mark.parametrize("name,args", [
    ("fill", (None, -1, C.c_float(0.0), None)),
    ("activate_array", (None, 4, 99, None)),
    ("gradient_array", (None, 4, -1, None, None)),
    ("bn_act_forward_train", (None, None, None, -1, 4, 4, None, None, None, None, None, None, 7, None)),
    ("bn_act_backward", (None, None, None, None, 2, 4, 4, None, None, None, None, None, None, None, None, 42, None)),
    ("forward_maxpool", (10, 4, 4, 1, 0, 2, 1, None, None, None, None)),
    ("shortcut", (1, 0, 4, 4, None, 4, 4, 4, C.c_float(1), C.c_float(1), None, None)),
    ("sgd_momentum", (16, None, None, C.c_float(0.1), C.c_float(0.9), C.c_float(5e-4), 128, None)),
    ("syncbn_forward_apply", (None, None, None, 2, 4, 4, None, 0, None, None, None, None, None, None, 7, None)),
    ("bn_act_forward_from_stats", (None, None, None, 2, 4, 4, None, 0, None, None, None, None, None, None, 7, None)),
    ("bn_act_forward_from_stats", (None, None, None, 2, 4, 4, None, 3, None, None, None, None, None, None, 99, None)),
])
def test_bad_arguments_are_rejected_without_a_device(built_lib, name, args):
    lib = _lib.lib()
    st = getattr(lib, "dnb_" + name)(*args)
    assert st == 1, (name, st, lib.dnb_last_error_detail())
    assert lib.dnb_last_error_detail()


def test_set_wait_limit_validates(built_lib):
    lib = _lib.lib()
    assert lib.dnb_set_wait_limit_ms(0) == 1
    assert lib.dnb_set_wait_limit_ms(2000) == 0


def test_call_refuses_a_wrong_argument_count(built_lib):
    # refused on the host before the library is entered
    with pytest.raises(TypeError, match="takes 4 arguments, 5 given"):
        _lib.call("fill", None, 4, C.c_float(0.0), None, None)
    with pytest.raises(TypeError, match="3 given"):
        _lib.call("fill", None, 4, C.c_float(0.0))
