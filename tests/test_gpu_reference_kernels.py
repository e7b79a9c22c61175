"""The reference's own GPU kernels as a second parity anchor, on the B200.

oracle/_ref/libref_gpu.so is the reference's src/kernels/darknet_kernels.hip compiled for
sm_100a with the reference's flags, launched with the reference's grids (oracle/ref_gpu.cu).
These tests run the reference's unfused GPU layer sequences and this library's fused entries
on the same bytes:

  * forward (convolutional.zig:263-268 + batchnorm.zig:129-153, 12 launches) against
    dnb_bn_act_forward_train: statistics within RTOL of each other relative to the norm of
    the summed terms (the two sum in different orders), rolling statistics, x_norm and y
    within RTOL / ATOL (the reference's GPU normalize divides by sqrt(var)+1e-6, the CPU
    restatement this library follows multiplies by its reciprocal);
  * backward (convolutional.zig:279-282 + batchnorm.zig:155-170, 7 launches) against
    dnb_bn_act_backward, both given the reference forward's y and statistics: the four
    per-channel vectors and dx within RTOL of each other relative to their term norms;
  * the weight SGD update (convolutional.zig:332-334, 3 launches) against
    dnb_sgd_momentum: bit-exact (both fuse a*x+y into one fma, as the reference's nvcc build
    contracts axpy).

Skipped when the library was not built (the reference tree was absent at build time)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu, synth
from parity import assert_bitexact, assert_close, channel_view

pytestmark = pytest.mark.gpu

SHAPES = [(4, 17, 53), (8, 16, 64), (16, 40, 196), (2, 3, 4), (128, 128, 1024)]


@pytest.fixture(scope="module")
def ref_gpu(cuda):
    from oracle.oracle import RefGpu

    try:
        return RefGpu()
    except FileNotFoundError as e:
        pytest.skip(str(e))


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def inputs(shape, seed):
    B, C, S = shape
    x = synth.normal(300 + seed, (B * C * S,), 0.2, 1.1)
    gamma = synth.uniform(301 + seed, (C,), 0.5, 1.5)
    beta = synth.normal(302 + seed, (C,), 0.0, 0.1)
    delta = synth.normal(303 + seed, (B * C * S,), 0.0, 1.0)
    rm = synth.normal(304 + seed, (C,), 0.0, 0.5)
    rv = synth.uniform(305 + seed, (C,), 0.5, 2.0)
    return x, gamma, beta, delta, rm, rv


def reference_forward(ref_gpu, x, gamma, beta, rm0, rv0, shape):
    B, C, S = shape
    out = dev(x)
    xs, xn = torch.empty_like(out), torch.empty_like(out)
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    rm, rv = dev(rm0), dev(rv0)
    g, b = dev(gamma), dev(beta)
    ref_gpu.conv_bn_forward(out.data_ptr(), xs.data_ptr(), xn.data_ptr(), mean.data_ptr(), var.data_ptr(),
                            rm.data_ptr(), rv.data_ptr(), g.data_ptr(), b.data_ptr(), B, C, S, gpu.LEAKY)
    return {k: host(v) for k, v in dict(y=out, x=xs, x_norm=xn, mean=mean, var=var, rm=rm, rv=rv).items()}


@pytest.mark.parametrize("shape", SHAPES)
def test_forward_matches_reference_gpu_sequence(ref_gpu, shape):
    B, C, S = shape
    x, gamma, beta, _, rm0, rv0 = inputs(shape, 0)
    ref = reference_forward(ref_gpu, x, gamma, beta, rm0, rv0, shape)
    assert_bitexact(ref["x"], x, "reference copy of x")

    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    xn = torch.empty_like(y)
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    rm, rv = dev(rm0), dev(rv0)
    gpu.bnActForwardTrain(dev(x), y, xn, B, C, S, dev(gamma), dev(beta), mean, var, rm, rv, gpu.LEAKY)
    gpu.check_device_error()

    n = B * S
    xv = channel_view(x, B, C, S).astype(np.float64)
    assert_close(host(mean), ref["mean"], "mean", scale=np.sqrt((xv * xv).sum(axis=1)) / n)
    dev2 = (xv - xv.mean(axis=1)[:, None]) ** 2
    vscale = np.sqrt((dev2 * dev2).sum(axis=1)) / max(n - 1, 1)
    assert_close(host(var), ref["var"], "variance", scale=vscale)
    assert_close(host(rm), ref["rm"], "rolling_mean", scale=np.sqrt((xv * xv).sum(axis=1)) / n)
    assert_close(host(rv), ref["rv"], "rolling_variance", scale=vscale)
    assert_close(host(xn), ref["x_norm"], "x_norm")
    assert_close(host(y), ref["y"], "y")


@pytest.mark.parametrize("shape", SHAPES)
def test_backward_matches_reference_gpu_sequence(ref_gpu, shape):
    B, C, S = shape
    x, gamma, beta, delta, rm0, rv0 = inputs(shape, 11)
    ref = reference_forward(ref_gpu, x, gamma, beta, rm0, rv0, shape)
    # both backwards get the reference forward's y (the leaky gate) and statistics
    yd, xd, xnd = dev(ref["y"]), dev(x), dev(ref["x_norm"])
    mean, var, gd = dev(ref["mean"]), dev(ref["var"]), dev(gamma)
    bu0 = synth.uniform(306, (C,), -1, 1)
    su0 = synth.uniform(307, (C,), -1, 1)

    d_ref = dev(delta)
    bu_r, su_r = dev(bu0), dev(su0)
    md_r, vd_r = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    ref_gpu.conv_bn_backward(yd.data_ptr(), d_ref.data_ptr(), xd.data_ptr(), xnd.data_ptr(), mean.data_ptr(),
                             var.data_ptr(), gd.data_ptr(), bu_r.data_ptr(), su_r.data_ptr(), md_r.data_ptr(),
                             vd_r.data_ptr(), B, C, S, gpu.LEAKY)

    dx = torch.empty_like(xd)
    bu, su = dev(bu0), dev(su0)
    md, vd = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    gpu.bnActBackward(xd, yd, dev(delta), dx, B, C, S, gd, dev(beta), mean, var, bu, su, md, vd, gpu.LEAKY)
    gpu.check_device_error()

    # term norms of each per-channel sum, from the reference's gated delta
    g = delta.copy()
    yv = ref["y"]
    g = np.where(yv > 0, g, g * np.float32(0.1)).astype(np.float32)
    gv = channel_view(g, B, C, S).astype(np.float64)
    xnv = channel_view(ref["x_norm"], B, C, S).astype(np.float64)
    v = ref["var"].astype(np.float64)
    gam = gamma.astype(np.float64)
    inv = 1.0 / np.sqrt(v + 1e-5)
    xm = channel_view(x, B, C, S).astype(np.float64) - ref["mean"].astype(np.float64)[:, None]
    n_bu = np.sqrt((gv * gv).sum(axis=1))
    n_su = np.sqrt(((gv * xnv) ** 2).sum(axis=1))
    n_md = n_bu * gam * inv
    n_vd = np.sqrt(((gv * xm) ** 2).sum(axis=1)) * gam * 0.5 * (v + 1e-5) ** -1.5
    assert_close(host(bu), host(bu_r), "bias_updates", atol=1e-6, scale=n_bu)
    assert_close(host(su), host(su_r), "scale_updates", atol=1e-6, scale=n_su)
    assert_close(host(md), host(md_r), "mean_delta", atol=1e-6, scale=n_md)
    assert_close(host(vd), host(vd_r), "variance_delta", atol=1e-6, scale=n_vd)
    # dx = g*gamma*inv + vd*2(x-mu)/n + md/n: bound by the magnitude of the three terms
    n = B * S
    md_h, vd_h = host(md_r).astype(np.float64), host(vd_r).astype(np.float64)
    t = (np.abs(gv * (gam * inv)[:, None]) + np.abs(vd_h[:, None] * 2 * xm / n) + np.abs(md_h / n)[:, None])
    scale = t.reshape(C, B, S).transpose(1, 0, 2).ravel()
    assert_close(host(dx), host(d_ref), "dx", scale=scale)


@pytest.mark.parametrize("n", [1, 1000, (1 << 20) + 3, 64 << 20])
def test_sgd_matches_reference_gpu_sequence_bitexact(ref_gpu, n):
    w0 = synth.normal(320, (n,), 0.0, 0.01)
    wu0 = synth.normal(321, (n,), 0.0, 1e-3)
    lr, momentum, decay, batch = 0.1, 0.9, 5e-4, 1024
    w_r, wu_r = dev(w0), dev(wu0)
    ref_gpu.sgd_weights(n, lr, momentum, decay, batch, w_r.data_ptr(), wu_r.data_ptr())
    w, wu = dev(w0), dev(wu0)
    gpu.sgdMomentum(n, w, wu, lr, momentum, decay, batch)
    gpu.check_device_error()
    assert_bitexact(host(w), host(w_r), "weights")
    assert_bitexact(host(wu), host(wu_r), "weight_updates")
