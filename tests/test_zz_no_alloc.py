"""dnb_mean_noalloc, the allocation-free per-channel mean, against dnb_mean through the C ABI.

Collected last (file name), so in a full run it comes after every other GPU test has used the
library's allocating entry points; `test_allocates_nothing_in_a_fresh_process` runs the
entry point in a new process that has loaded nothing else, and checks through
cudaMemGetInfo (dnb_mem_info) that repeated calls leave the device's free memory unchanged
while one call of the allocating dnb_mean does not."""
from __future__ import annotations

import json
import os
import subprocess
import sys
import textwrap

import numpy as np
import pytest
import torch

from darknet_zig_b200 import _lib, gpu, synth
from parity import ATOL, RTOL, assert_close, exact_channel_sum

pytestmark = pytest.mark.gpu

SCRATCH_FLOATS = 1 << 18  # the fixed partial-sum array in csrc/dnb_reduce.cu
CHUNK = 32768             # elements one partial covers


def mean_noalloc(x, batch, filters, spatial, out):
    _lib.call("mean_noalloc", gpu._p(x), int(batch), int(filters), int(spatial), gpu._p(out), gpu._s())


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


# (batch, filters, spatial) pairs run back to back: the second call of each pair reuses the
# array the first one left its partials in (a shrinking, a growing and a ragged pair)
PAIRS = [
    ((16, 40, 196), (8, 16, 64)),
    ((2, 3, 4), (64, 64, 3136)),
    ((4, 17, 53), (3, 5, 7)),
]


@pytest.mark.parametrize("first,second", PAIRS)
def test_two_calls_in_a_row_match_dnb_mean(cuda, first, second):
    xs = [synth.normal(500 + i, (b * c * s,), 0.5, 1.0) for i, (b, c, s) in enumerate((first, second))]
    got = []
    for x, (b, c, s) in zip(xs, (first, second)):
        out = torch.full((c,), float("nan"), device=cuda)
        mean_noalloc(torch.from_numpy(x).to(cuda), b, c, s, out)
        got.append(host(out))
    for x, (b, c, s), g in zip(xs, (first, second), got):
        want = torch.empty(c, device=cuda)
        gpu.mean(torch.from_numpy(x).to(cuda), b, c, s, want)
        want = host(want)
        assert_close(g, want, "mean_noalloc vs dnb_mean", rtol=RTOL, atol=ATOL)
        exact, norm = exact_channel_sum(x, b, c, s)
        assert_close(g, exact / (b * s), "mean_noalloc vs exact", scale=norm / (b * s))


def test_ragged_chunks_then_oversize_is_rejected(cuda):
    # 4096 channels of 32769 elements: two partials per channel, the second of one element
    batch, filters, spatial = 1, 4096, CHUNK + 1
    x = synth.uniform(510, (batch * filters * spatial,), -1.0, 3.0)
    xd = torch.from_numpy(x).to(cuda)
    out = torch.empty(filters, device=cuda)
    mean_noalloc(xd, batch, filters, spatial, out)
    want = torch.empty(filters, device=cuda)
    gpu.mean(xd, batch, filters, spatial, want)
    assert_close(host(out), host(want), "ragged mean_noalloc vs dnb_mean")
    # 65535 channels x 5 partials > 262144: refused on the host before any launch
    small = torch.zeros(4, device=cuda)
    with pytest.raises(_lib.DnbError) as e:
        mean_noalloc(small, 1, 65535, 4 * CHUNK + 1, torch.empty(65535, device=cuda))
    assert e.value.status == 5 and "fixed scratch" in str(e.value)
    # a refused call leaves the entry point usable
    mean_noalloc(xd, batch, filters, spatial, out)
    assert_close(host(out), host(want), "mean_noalloc after a refusal")


_CHILD = textwrap.dedent("""
    import ctypes as C, json, sys
    import numpy as np
    sys.path.insert(0, sys.argv[1])
    from darknet_zig_b200 import _lib
    from darknet_zig_b200._lib import call
    L = _lib.lib()
    call("init", 0)
    B, F, S = 16, 40, 196
    x = np.arange(B * F * S, dtype=np.float32) % 7 - 3
    def dalloc(n):
        p = C.c_void_p()
        call("malloc", C.byref(p), n)
        return p.value
    xd, o1, o2 = dalloc(x.nbytes), dalloc(4 * F), dalloc(4 * F)
    call("push", xd, x.ctypes.data, x.nbytes, None)
    call("sync")
    def free():
        f, t = C.c_size_t(), C.c_size_t()
        call("sync")
        call("mem_info", C.byref(f), C.byref(t))
        return f.value
    call("mean_noalloc", xd, B, F, S, o1, None)  # first call on the device: its set-up
    f0 = free()
    for _ in range(3):
        call("mean_noalloc", xd, B, F, S, o1, None)
    f1 = free()
    call("mean", xd, B, F, S, o2, None)  # allocates this stream's workspace
    f2 = free()
    a, b = np.empty(F, np.float32), np.empty(F, np.float32)
    call("pull", a.ctypes.data, o1, 4 * F, None)
    call("pull", b.ctypes.data, o2, 4 * F, None)
    call("sync")
    print(json.dumps({"free_after_setup": f0, "free_after_calls": f1, "free_after_dnb_mean": f2,
                      "max_abs_diff": float(np.max(np.abs(a - b)))}))
""")


def test_allocates_nothing_in_a_fresh_process(built_lib):
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    r = subprocess.run([sys.executable, "-c", _CHILD, root], capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr[-3000:]
    d = json.loads(r.stdout.strip().splitlines()[-1])
    assert d["free_after_calls"] == d["free_after_setup"], d
    assert d["free_after_dnb_mean"] < d["free_after_calls"], d  # the measurement sees an allocation
    assert d["max_abs_diff"] <= 1e-6, d
