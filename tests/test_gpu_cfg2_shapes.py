"""GPU parity at BASELINE config 2's real shapes: the inference-mode fused BN + leaky sweep
over the tiny-classifier stack at batch 64, and the 2x2 / stride-2 maxpool with argmax
indices between its stages, each bit-exact against the CPU restatement of the reference
(batchnorm.zig:148 -> blas.normalize / scaleBias / addBias, activations.zig; pooling.zig:59-93).

Inputs follow the config: x ~ N(0, 1), gamma ~ U(0.5, 1.5), beta ~ N(0, 0.1), rolling
variance ~ U(0.5, 2), rolling mean ~ N(0, 0.5), seeded per stage (the per-channel vectors from
the package's documented generator, the large x from torch's seeded CUDA generator, which is
far faster at these sizes; oracle and kernel read the same bytes). These sizes (up to 51.4 M
elements, 205 MB per tensor) run the kernels' full-size index paths, including the 14 x 14
stage whose width is not a multiple of 4."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu, synth
from parity import assert_bitexact

pytestmark = pytest.mark.gpu

N = 64
STAGES = [(16, 224), (32, 112), (64, 56), (128, 28), (256, 14), (512, 7), (1024, 7)]


def big_normal(seed, n):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    t = torch.randn(n, generator=g, device="cuda")
    return t, host(t).copy()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("c,hw", STAGES, ids=[f"{c}x{hw}x{hw}" for c, hw in STAGES])
def test_bn_act_forward_infer_cfg2(cuda, oracle, c, hw):
    S = hw * hw
    E = N * c * S
    seed = 3000 + c
    xd, x = big_normal(seed, E)
    gamma = synth.uniform(seed + 1, (c,), 0.5, 1.5)
    beta = synth.normal(seed + 2, (c,), 0.0, 0.1)
    rmean = synth.normal(seed + 3, (c,), 0.0, 0.5)
    rvar = synth.uniform(seed + 4, (c,), 0.5, 2.0)
    d = lambda a: torch.from_numpy(a).cuda()  # noqa: E731
    y = torch.empty(E, dtype=torch.float32, device="cuda")
    gpu.bnActForwardInfer(xd, y, N, c, S, d(gamma), d(beta), d(rmean), d(rvar), gpu.LEAKY)
    got = host(y)
    want = x  # in place on the host copy
    oracle.normalize(want, rmean, rvar, N, c, S)
    oracle.scale_bias(want, gamma, N, c, S)
    oracle.add_bias(want, beta, N, c, S)
    oracle.activate_array(want, gpu.LEAKY)
    assert_bitexact(got, want, f"bn_act_forward_infer 64x{c}x{hw}x{hw}")


@pytest.mark.parametrize("c,hw", STAGES[:5], ids=[f"{c}x{hw}x{hw}" for c, hw in STAGES[:5]])
def test_maxpool_cfg2(cuda, oracle, c, hw):
    E = N * c * hw * hw
    size, stride, pad = 2, 2, 1  # [maxpool] size=2 stride=2, pad defaulting to size-1 (parser.zig:168)
    oh = oracle.maxpool_out_dim(hw, size, stride, pad)
    On = N * c * oh * oh
    xd, x = big_normal(4000 + c, E)
    out = torch.empty(On, dtype=torch.float32, device="cuda")
    idx = torch.empty(On, dtype=torch.int32, device="cuda")
    gpu.forwardMaxpool(On, hw, hw, c, stride, size, pad, xd, out, idx)
    w_out = np.zeros(On, np.float32)
    w_idx = np.zeros(On, np.int32)
    oracle.forward_maxpool(N, hw, hw, c, stride, size, pad, x, w_out, w_idx)
    assert_bitexact(host(out), w_out, f"maxpool values 64x{c}x{hw}x{hw}")
    got_idx = host(idx)
    bad = np.flatnonzero(got_idx != w_idx)
    assert bad.size == 0, f"maxpool indices: {bad.size} differ, first at {bad[0]}: {got_idx[bad[0]]} vs {w_idx[bad[0]]}"
