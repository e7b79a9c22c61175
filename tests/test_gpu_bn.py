"""GPU parity of batchnorm + activation: the fused forward/backward kernels (persistent and
generic paths), the standalone per-channel reductions, and the reference's unfused op
sequence through the per-op ABI.

Checks per call:
  * per-channel statistics and sums: within RTOL/ATOL of the float64 sum of the same
    float32 terms (relative to max(|exact|, ||terms||_2), see parity.py), and within the
    same bar of the reference CPU restatement widened by that restatement's own error;
  * every per-element output: bit-identical to the CPU restatement run with the
    per-channel statistics the kernel produced;
  * rolling statistics: bit-identical to scal(0.99) + axpy(0.01) of the kernel's stats.
"""
from __future__ import annotations

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu, synth
from darknet_zig_b200.layers import BatchNorm
from parity import assert_bitexact, assert_close, channel_view, exact_channel_sum

# bias_updates / scale_updates accumulate into the caller's values: one float32 rounding of
# a result of magnitude ~1 (the initial values are U(-1, 1)) is up to 6e-8, below this bar
ACC_ATOL = 1e-6

pytestmark = pytest.mark.gpu

# (batch, filters, spatial): generic path (S % 4 != 0), persistent path at several unit
# shapes, the gputest shape, and the BASELINE configs 0/1 and 4 (per GPU) plus a 32 MiB
# single-group forward
SHAPES = [
    (4, 17, 53),
    (8, 16, 64),
    (2, 3, 4),
    (16, 40, 196),
    (5, 7, 28),
    (64, 64, 3136),
    (1, 300, 100),
]
FULL_SHAPES = [(128, 128, 1024), (128, 256, 784), (64, 128, 1024)]


# The fused entries pick, in order: the channel-per-CTA kernel for small channels, the L2
# sweep, the cluster-per-channel kernel, the grid-wide shared-memory-staged kernel, and the
# generic multi-launch path. The library reads these switches at every call, so each test
# below runs each path on the same inputs ("default" is the order itself).
BN_PATHS = {
    "default": {},
    "sweep": {"DNB_BN_SMALL": "0", "DNB_BN_CLUSTER": "0", "DNB_BN_STAGE": "0"},
    # the sweep with its streaming warps split into statistics readers and output writers (the
    # default only for backwards over many channel groups)
    "sweep-split": {"DNB_BN_SMALL": "0", "DNB_BN_CLUSTER": "0", "DNB_BN_STAGE": "0", "DNB_BN_SPLIT": "7"},
    "cluster": {"DNB_BN_SMALL": "0", "DNB_BN_SWEEP": "0"},
    "stage": {"DNB_BN_SMALL": "0", "DNB_BN_CLUSTER": "0", "DNB_BN_SWEEP": "0"},
    "generic": {"DNB_BN_PERSISTENT": "0"},
}


@pytest.fixture(params=list(BN_PATHS))
def bn_path(request, monkeypatch):
    for k, v in BN_PATHS[request.param].items():
        monkeypatch.setenv(k, v)
    return request.param


def dev(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def make_inputs(shape, seed=0, mean_shift=0.0):
    B, C, S = shape
    x = synth.normal(100 + seed, (B * C * S,), mean_shift, 1.0)
    gamma = synth.uniform(101 + seed, (C,), 0.5, 1.5)
    beta = synth.normal(102 + seed, (C,), 0.0, 0.1)
    delta = synth.normal(103 + seed, (B * C * S,), 0.0, 1.0)
    rm = synth.normal(104 + seed, (C,), 0.0, 0.5)
    rv = synth.uniform(105 + seed, (C,), 0.5, 2.0)
    return x, gamma, beta, delta, rm, rv


def oracle_bn_apply(oracle, x, mean, var, gamma, beta, shape, act):
    """normalize -> scaleBias -> addBias -> activate with given statistics (batchnorm.zig:145-152)."""
    B, C, S = shape
    xn = x.copy()
    oracle.normalize(xn, mean, var, B, C, S)
    y = xn.copy()
    oracle.scale_bias(y, gamma, B, C, S)
    oracle.add_bias(y, beta, B, C, S)
    oracle.activate_array(y, act)
    return xn, y


def check_forward_stats(oracle, x, shape, mean_got, var_got):
    B, C, S = shape
    n = B * S
    xv = channel_view(x, B, C, S).astype(np.float64)
    m_exact = xv.mean(axis=1)
    assert_close(mean_got, m_exact, "mean", scale=np.sqrt((xv * xv).sum(axis=1)) / n)
    dev2 = (xv - m_exact[:, None]) ** 2
    v_exact = dev2.sum(axis=1) / (n - 1)
    assert_close(var_got, v_exact, "variance", scale=np.sqrt((dev2 * dev2).sum(axis=1)) / (n - 1))
    # the reference's own fp32 sequential statistics, allowed their own error
    m_ref = np.zeros(C, np.float32)
    v_ref = np.zeros(C, np.float32)
    oracle.mean(x, B, C, S, m_ref)
    oracle.variance(x, m_ref, B, C, S, v_ref)
    own = np.abs(v_ref.astype(np.float64) - v_exact)
    assert_close(var_got, v_ref, "variance vs reference", atol=1e-6 + own)


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("act", [gpu.LEAKY, gpu.RELU, gpu.LINEAR, gpu.LOGISTIC])
def test_fused_forward_train(cuda, oracle, shape, act, bn_path):
    B, C, S = shape
    x, gamma, beta, _, rm0, rv0 = make_inputs(shape)
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    xn = torch.empty_like(y)
    mean = torch.zeros(C, device="cuda")
    var = torch.zeros(C, device="cuda")
    rm = dev(rm0)
    rv = dev(rv0)
    gpu.bnActForwardTrain(dev(x), y, xn, B, C, S, dev(gamma), dev(beta), mean, var, rm, rv, act)
    m_got, v_got = host(mean), host(var)
    check_forward_stats(oracle, x, shape, m_got, v_got)
    # rolling stats: scal(0.99) + axpy(1-0.99) of the kernel's own statistics
    rm_w, rv_w = rm0.copy(), rv0.copy()
    oracle.scal(0.99, rm_w)
    oracle.axpy(np.float32(1) - np.float32(0.99), m_got, rm_w)
    oracle.scal(0.99, rv_w)
    oracle.axpy(np.float32(1) - np.float32(0.99), v_got, rv_w)
    assert_bitexact(host(rm), rm_w, "rolling_mean")
    assert_bitexact(host(rv), rv_w, "rolling_variance")
    xn_w, y_w = oracle_bn_apply(oracle, x, m_got, v_got, gamma, beta, shape, act)
    assert_bitexact(host(xn), xn_w, "x_norm")
    if act == gpu.LOGISTIC:  # CUDA expf vs libm expf
        assert_close(host(y), y_w, "y", rtol=1e-5, atol=1e-6)
    else:
        assert_bitexact(host(y), y_w, "y")


def oracle_backward_given_stats(oracle, x, y, delta, shape, gamma, mean, var, md, vd, act):
    """gradient -> scaleBias -> normalizeDelta with the kernel's mean_delta/variance_delta."""
    B, C, S = shape
    g = delta.copy()
    oracle.gradient_array(y, act, g)
    gs = g.copy()
    oracle.scale_bias(gs, gamma, B, C, S)
    dx = gs.copy()
    oracle.normalize_delta(x, mean, var, md, vd, B, C, S, dx)
    return g, gs, dx


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("act", [gpu.LEAKY, gpu.RELU, gpu.LINEAR, gpu.LOGISTIC])
@pytest.mark.parametrize("with_y", [False, True])
def test_fused_backward(cuda, oracle, shape, act, with_y, bn_path):
    B, C, S = shape
    x, gamma, beta, delta, _, _ = make_inputs(shape, seed=7)
    # forward first (fused) to get the statistics and y the backward uses
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    mean = torch.zeros(C, device="cuda")
    var = torch.zeros(C, device="cuda")
    gpu.bnActForwardTrain(dev(x), y, None, B, C, S, dev(gamma), dev(beta), mean, var, torch.zeros(C, device="cuda"),
                          torch.zeros(C, device="cuda"), act)
    m, v, y_h = host(mean), host(var), host(y)
    bu0 = synth.uniform(200, (C,), -1, 1)
    su0 = synth.uniform(201, (C,), -1, 1)
    bu, su = dev(bu0), dev(su0)
    md = torch.zeros(C, device="cuda")
    vd = torch.zeros(C, device="cuda")
    dxt = torch.empty_like(y)
    gpu.bnActBackward(dev(x), y if with_y else None, dev(delta), dxt, B, C, S, dev(gamma), dev(beta), mean, var, bu,
                      su, md, vd, act)
    md_h, vd_h = host(md), host(vd)
    g, gs, dx_w = oracle_backward_given_stats(oracle, x, y_h, delta, shape, gamma, m, v, md_h, vd_h, act)
    # bit-exact for every activation: without y the kernel recomputes y from x with the
    # forward's own arithmetic (CUDA expf included), so it equals the stored device y
    assert_bitexact(host(dxt), dx_w, "dx")
    # per-channel sums against float64 sums of the same float32 terms (bu and su also
    # carry one float32 rounding of the accumulation into the caller's initial values)
    s1, s1n = exact_channel_sum(g, B, C, S)
    assert_close(host(bu) - bu0, s1, "bias_updates", atol=ACC_ATOL, scale=s1n)
    xn = x.copy()
    oracle.normalize(xn, m, v, B, C, S)
    s2, s2n = exact_channel_sum(g * xn, B, C, S)
    assert_close(host(su) - su0, s2, "scale_updates", atol=ACC_ATOL, scale=s2n)
    inv = (-1.0 / np.sqrt(v.astype(np.float32) + np.float32(1e-5))).astype(np.float64)
    sgs, sgsn = exact_channel_sum(gs, B, C, S)
    assert_close(md_h, sgs * inv, "mean_delta", scale=sgsn * np.abs(inv))
    fac = -0.5 * (v.astype(np.float64) + 1e-5) ** -1.5
    xm = (x.reshape(B, C, S) - m[None, :, None]).ravel().astype(np.float32)
    svd, svdn = exact_channel_sum(gs * xm, B, C, S)
    assert_close(vd_h, svd * fac, "variance_delta", scale=svdn * np.abs(fac))


@pytest.mark.parametrize("shape", [(8, 16, 64), (16, 40, 196), (32, 64, 784), (4, 17, 53)])
@pytest.mark.parametrize("act", [gpu.LEAKY, gpu.LINEAR])
def test_fused_backward_edge_numerators(cuda, oracle, shape, act, bn_path):
    """normalize_delta divides vd * 2 * (x - mean) by the element count (blas.zig:200); the
    kernels replace the division by a verified two-operation form for numerators in its
    range and divide the rest. Channels here make numerators of +0 and -0 (a constant
    channel, elements equal to their channel's exact mean), tiny ones (delta ~ 1e-30) and
    large ones (delta ~ 1e20): dx must still equal the reference's IEEE division bit for bit."""
    B, C, S = shape
    x, gamma, beta, delta, _, _ = make_inputs(shape, seed=11)
    xv = x.reshape(B, C, S)
    dv = delta.reshape(B, C, S)
    xv[:, 0, :] = 1.5                                              # constant: x - mean = 0
    xv[:, 1, :] = np.resize(np.float32([1.0, 1.5, 1.5, 2.0]), (B, S))  # mean 1.5: zeros where x = 1.5
    dv[:, 2, :] = 0.0                                              # vd = 0
    dv[:, 3, :] *= np.float32(1e-30)                               # tiny numerators
    dv[:, 4 % C, :] *= np.float32(1e20)                            # large numerators
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    mean = torch.zeros(C, device="cuda")
    var = torch.zeros(C, device="cuda")
    gpu.bnActForwardTrain(dev(x), y, None, B, C, S, dev(gamma), dev(beta), mean, var, torch.zeros(C, device="cuda"),
                          torch.zeros(C, device="cuda"), act)
    m, v, y_h = host(mean), host(var), host(y)
    assert m[0] == np.float32(1.5)  # the constant channel's numerators are all zero
    md = torch.zeros(C, device="cuda")
    vd = torch.zeros(C, device="cuda")
    bu, su = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    dxt = torch.empty_like(y)
    gpu.bnActBackward(dev(x), None, dev(delta), dxt, B, C, S, dev(gamma), dev(beta), mean, var, bu, su, md, vd, act)
    md_h, vd_h = host(md), host(vd)
    _, _, dx_w = oracle_backward_given_stats(oracle, x, y_h, delta, shape, gamma, m, v, md_h, vd_h, act)
    assert_bitexact(host(dxt), dx_w, "dx")


def backward_sum_scales(oracle, x, y, delta, gamma, m, v, shape, act):
    """Per-channel 2-norms of the terms behind bias_updates, scale_updates, mean_delta and
    variance_delta (the scale of the reduction bar, parity.py)."""
    B, C, S = shape
    g = delta.copy()
    oracle.gradient_array(y, act, g)
    gs = g.copy()
    oracle.scale_bias(gs, gamma, B, C, S)
    xn = x.copy()
    oracle.normalize(xn, m, v, B, C, S)
    xm = (x.reshape(B, C, S) - m[None, :, None]).ravel().astype(np.float32)
    inv = 1.0 / np.sqrt(v.astype(np.float64) + 1e-5)
    fac = 0.5 * (v.astype(np.float64) + 1e-5) ** -1.5
    return {"bu": exact_channel_sum(g, B, C, S)[1], "su": exact_channel_sum(g * xn, B, C, S)[1],
            "md": exact_channel_sum(gs, B, C, S)[1] * inv, "vd": exact_channel_sum(gs * xm, B, C, S)[1] * fac}


@pytest.mark.slow
@pytest.mark.parametrize("shape", FULL_SHAPES)
def test_fused_full_size_forward_backward(cuda, oracle, shape, bn_path):
    """BASELINE configs 0/1 (128x128x32x32) and 4 (per GPU 128x256x28x28), leaky 0.1, and a
    32 MiB tensor whose forward plan is a single channel group."""
    test_fused_forward_train(cuda, oracle, shape, gpu.LEAKY, bn_path)
    test_fused_backward(cuda, oracle, shape, gpu.LEAKY, False, bn_path)


@pytest.mark.parametrize("shape", [(8, 16, 64), (2, 3, 4), (16, 40, 196), (1, 300, 100), (128, 128, 1024),
                                   (128, 256, 784), (64, 1024, 49), (16, 40, 169), (4, 17, 53)])
def test_fused_entries_are_one_launch(cuda, shape):
    """With aligned tensors each fused entry is a single kernel launch (the staged kernel),
    not the multi-launch generic path: spatial % 4 == 0, and also spatial % 4 != 0 (7x7,
    13x13, 53) whenever the element count is a multiple of 4."""
    B, C, S = shape
    x, gamma, beta, delta, rm0, rv0 = make_inputs(shape, seed=5)
    y = torch.empty(x.size, dtype=torch.float32, device="cuda")
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    xd, gd, bd, rm, rv = dev(x), dev(gamma), dev(beta), dev(rm0), dev(rv0)
    n0 = gpu.launch_count()
    gpu.bnActForwardTrain(xd, y, None, B, C, S, gd, bd, mean, var, rm, rv, gpu.LEAKY)
    n1 = gpu.launch_count()
    dx = torch.empty_like(y)
    bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(4))
    dd = dev(delta)
    n2 = gpu.launch_count()
    gpu.bnActBackward(xd, None, dd, dx, B, C, S, gd, bd, mean, var, bu, su, md, vd, gpu.LEAKY)
    n3 = gpu.launch_count()
    torch.cuda.synchronize()
    gpu.check_device_error()
    assert (n1 - n0, n3 - n2) == (1, 1)


@pytest.mark.parametrize("shape", [(8, 16, 64), (4, 17, 53), (128, 128, 1024)])
def test_fused_is_deterministic(cuda, shape):
    B, C, S = shape
    x, gamma, beta, delta, rm0, rv0 = make_inputs(shape, seed=3)
    outs = []
    for _ in range(2):
        y = torch.empty(x.size, dtype=torch.float32, device="cuda")
        mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
        gpu.bnActForwardTrain(dev(x), y, None, B, C, S, dev(gamma), dev(beta), mean, var, dev(rm0), dev(rv0),
                              gpu.LEAKY)
        dx = torch.empty_like(y)
        bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(4))
        gpu.bnActBackward(dev(x), None, dev(delta), dx, B, C, S, dev(gamma), dev(beta), mean, var, bu, su, md, vd,
                          gpu.LEAKY)
        outs.append([host(t) for t in (y, mean, var, dx, bu, su, md, vd)])
    for a, b in zip(outs[0], outs[1]):
        assert_bitexact(a, b, "second run")


@pytest.mark.parametrize("shape", [(4, 17, 53), (8, 16, 64), (3, 5, 2)])
def test_standalone_reductions(cuda, oracle, shape):
    B, C, S = shape
    x, _, _, delta, _, rv = make_inputs(shape, seed=11)
    mean = np.zeros(C, np.float32)
    oracle.mean(x, B, C, S, mean)
    xn = x.copy()
    oracle.normalize(xn, mean, rv, B, C, S)

    out = torch.zeros(C, device="cuda")
    gpu.mean(dev(x), B, C, S, out)
    s, sn = exact_channel_sum(x, B, C, S)
    scale_f = np.float32(1) / np.float32(B * S)
    assert_close(host(out), s * scale_f, "mean", scale=sn * scale_f)

    out = torch.zeros(C, device="cuda")
    gpu.variance(dev(x), dev(mean), B, C, S, out)
    d2 = ((x.reshape(B, C, S) - mean[None, :, None]) ** 2).ravel().astype(np.float32)
    s, sn = exact_channel_sum(d2, B, C, S)
    sf = np.float32(1) / np.float32(B * S - 1)
    assert_close(host(out), s * sf, "variance", scale=sn * sf)

    bu0 = synth.uniform(12, (C,), -1, 1)
    out = dev(bu0)
    gpu.backwardBias(out, dev(delta), B, C, S)
    s, sn = exact_channel_sum(delta, B, C, S)
    assert_close(host(out) - bu0, s, "backward_bias", atol=1e-6, scale=sn)

    out = dev(bu0)
    gpu.backwardScale(dev(xn), dev(delta), B, C, S, out)
    s, sn = exact_channel_sum(delta * xn, B, C, S)
    assert_close(host(out) - bu0, s, "backward_scale", atol=1e-6, scale=sn)

    out = torch.zeros(C, device="cuda")
    gpu.meanDelta(dev(delta), dev(rv), B, C, S, out)
    s, sn = exact_channel_sum(delta, B, C, S)
    f = (np.float32(-1) / np.sqrt(rv + np.float32(1e-5))).astype(np.float64)
    assert_close(host(out), s * f, "mean_delta", atol=1e-6, scale=sn * np.abs(f))

    out = torch.zeros(C, device="cuda")
    gpu.varianceDelta(dev(x), dev(delta), dev(mean), dev(rv), B, C, S, out)
    xm = (x.reshape(B, C, S) - mean[None, :, None]).ravel().astype(np.float32)
    s, sn = exact_channel_sum(delta * xm, B, C, S)
    f = -0.5 * (rv.astype(np.float64) + 1e-5) ** -1.5
    assert_close(host(out), s * f, "variance_delta", atol=1e-6, scale=sn * np.abs(f))


@pytest.mark.parametrize("shape", [(4, 17, 53), (8, 16, 64), (16, 40, 196)])
def test_unfused_reference_sequence_matches_fused(cuda, oracle, shape):
    """The reference's own launch sequence (batchnorm.zig:129-174 through the per-op ABI)
    and the fused kernels agree within the reduction bar."""
    B, C, S = shape
    x, gamma, beta, delta, _, _ = make_inputs(shape, seed=21)
    layers = []
    for fused in (True, False):
        bn = BatchNorm(B, C, 1, S, gpu.LEAKY)
        bn.scales.copy_(dev(gamma))
        bn.biases.copy_(dev(beta))
        y = bn.forward(dev(x).reshape(B, C, 1, S), train=True, fused=fused)
        d = dev(delta).reshape(B, C, 1, S).clone()
        dx = bn.backward(d, train=True, fused=fused)
        layers.append({k: host(v) for k, v in dict(y=y, dx=dx, mean=bn.mean, variance=bn.variance,
                                                   rm=bn.rolling_mean, rv=bn.rolling_variance,
                                                   bu=bn.bias_updates, su=bn.scale_updates, md=bn.mean_delta,
                                                   vd=bn.variance_delta).items()})
    f, u = layers
    for k in ("y", "mean", "variance", "rm", "rv", "dx"):
        assert_close(f[k], u[k], k)
    # the reductions: relative to the per-channel terms' 2-norm, as every reduction here
    sc = backward_sum_scales(oracle, x, f["y"], delta, gamma, f["mean"], f["variance"], shape, gpu.LEAKY)
    for k in ("bu", "su", "md", "vd"):
        assert_close(f[k], u[k], k, scale=sc[k])


def test_syncbn_split_path_two_shards_on_one_gpu(cuda, oracle):
    """Split sync-BN API: two half-batch shards, partials combined as an all-gather would,
    give the statistics and outputs of the whole batch in one shard."""
    from darknet_zig_b200._lib import call

    B, C, S = 16, 24, 196
    x, gamma, beta, delta, _, _ = make_inputs((B, C, S), seed=31)
    h = B // 2
    g_d, b_d = dev(gamma), dev(beta)  # held: the ABI takes raw pointers
    xs = [dev(x[: h * C * S]), dev(x[h * C * S:])]
    parts = [torch.zeros(C, 2, dtype=torch.float64, device="cuda") for _ in range(2)]
    stream = torch.cuda.current_stream().cuda_stream
    for xi, p in zip(xs, parts):
        call("syncbn_forward_partials", xi.data_ptr(), h, C, S, p.data_ptr(), stream)
    gathered = torch.stack(parts).contiguous()
    m_full, v_full = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    y_full = torch.empty(B * C * S, device="cuda")
    gpu.bnActForwardTrain(dev(x), y_full, None, B, C, S, g_d, b_d, m_full, v_full, torch.zeros(C, device="cuda"),
                          torch.zeros(C, device="cuda"), gpu.LEAKY)
    for i, xi in enumerate(xs):
        y = torch.empty(h * C * S, device="cuda")
        m, v, rm, rv = (torch.zeros(C, device="cuda") for _ in range(4))
        call("syncbn_forward_apply", xi.data_ptr(), y.data_ptr(), None, h, C, S, gathered.data_ptr(), 2,
             g_d.data_ptr(), b_d.data_ptr(), m.data_ptr(), v.data_ptr(), rm.data_ptr(), rv.data_ptr(), gpu.LEAKY,
             stream)
        assert_close(host(m), host(m_full), "sync mean")
        assert_close(host(v), host(v_full), "sync variance")
        half = slice(i * h * C * S, (i + 1) * h * C * S)
        assert_close(host(y), host(y_full)[half], "sync y")
    # backward: partial sums of both shards, summed as an all-reduce would
    d_d = dev(delta)
    ds = [d_d[: h * C * S], d_d[h * C * S:]]
    bparts = [torch.zeros(C, 2, dtype=torch.float64, device="cuda") for _ in range(2)]
    for xi, di, p in zip(xs, ds, bparts):
        call("syncbn_backward_partials", xi.data_ptr(), None, di.data_ptr(), h, C, S, g_d.data_ptr(), b_d.data_ptr(),
             m_full.data_ptr(), v_full.data_ptr(), gpu.LEAKY, p.data_ptr(), stream)
    red = (bparts[0] + bparts[1]).contiguous()
    dx_full = torch.empty_like(y_full)
    bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(4))
    gpu.bnActBackward(dev(x), None, d_d, dx_full, B, C, S, g_d, b_d, m_full, v_full, bu, su, md, vd, gpu.LEAKY)
    sc = backward_sum_scales(oracle, x, host(y_full), delta, gamma, host(m_full), host(v_full), (B, C, S),
                             gpu.LEAKY)
    for i, (xi, di) in enumerate(zip(xs, ds)):
        dx = torch.empty(h * C * S, device="cuda")
        bu2, su2, md2, vd2 = (torch.zeros(C, device="cuda") for _ in range(4))
        call("syncbn_backward_apply", xi.data_ptr(), None, di.data_ptr(), dx.data_ptr(), h, C, S, B * S,
             red.data_ptr(), g_d.data_ptr(), b_d.data_ptr(), m_full.data_ptr(), v_full.data_ptr(), bu2.data_ptr(),
             su2.data_ptr(), md2.data_ptr(), vd2.data_ptr(), gpu.LEAKY, stream)
        for got, want, name, k in ((bu2, bu, "bias_updates", "bu"), (su2, su, "scale_updates", "su"),
                                   (md2, md, "mean_delta", "md"), (vd2, vd, "variance_delta", "vd")):
            assert_close(host(got), host(want), f"sync {name}", scale=sc[k])
        half = slice(i * h * C * S, (i + 1) * h * C * S)
        assert_close(host(dx), host(dx_full)[half], "sync dx")


def test_rolling_statistics_survive_a_weights_round_trip(cuda, tmp_path):
    """Rolling statistics produced by the fused training forward, saved in the reference's
    .weights layout (parser.zig:535-543) and loaded into a fresh layer, give a bit-identical
    inference forward."""
    from darknet_zig_b200 import weights

    B, C, H, W = 8, 16, 8, 8
    bn = BatchNorm(B, C, H, W)
    bn.scales.copy_(dev(synth.uniform(40, (C,), 0.5, 1.5)))
    bn.biases.copy_(dev(synth.normal(41, (C,), 0.0, 0.1)))
    for k in range(3):
        bn.forward(dev(synth.normal(42 + k, (B * C * H * W,), 0.3, 1.2)), train=True)
    x_test = dev(synth.normal(50, (B * C * H * W,), 0.0, 1.0))
    y_before = host(bn.forward(x_test, train=False))
    assert host(bn.rolling_variance).any()
    path = str(tmp_path / "bn.weights")
    p = weights.batchnorm_params(bn, kind="convolutional", nweights=C * 4 * 9)
    p.pull()
    weights.save(path, [p], seen=24)
    fresh = BatchNorm(B, C, H, W)
    q = weights.batchnorm_params(fresh, kind="convolutional", nweights=C * 4 * 9)
    assert weights.load(path, [q]) == 24
    q.push()
    for name in ("scales", "biases", "rolling_mean", "rolling_variance"):
        assert_bitexact(host(getattr(fresh, name)), host(getattr(bn, name)), name)
    assert_bitexact(host(fresh.forward(x_test, train=False)), y_before, "inference output")
