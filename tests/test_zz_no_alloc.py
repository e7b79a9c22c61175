"""dnb_mean_noalloc, the allocation-free per-channel mean, against dnb_mean through the C ABI.

Collected last (file name) so that it runs both on a fresh process and after every other
GPU test has used the library's allocating entry points."""
from __future__ import annotations

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
