"""GPU parity: elementwise, broadcast, pooling, softmax, shortcut and SGD ops through the
C ABI against the CPU oracle on the same seeded inputs."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu, synth
from parity import assert_bitexact, assert_close

pytestmark = pytest.mark.gpu

SIZES = [0, 1, 3, 4, 5, 255, 4099, (1 << 20) + 3]
EXACT_ACTS = [gpu.LEAKY, gpu.RELU, gpu.LINEAR, gpu.RELIE, gpu.RAMP, gpu.PLSE, gpu.STAIR, gpu.HARDTAN, gpu.LHTAN]
EXP_ACTS = [gpu.LOGISTIC, gpu.LOGGY, gpu.ELU, gpu.SELU, gpu.TANH]  # CUDA expf vs libm expf


def dev(a, offset=0):
    """Device copy; offset > 0 places it `offset` floats into a larger buffer so that the
    pointer is not 16-byte aligned (exercises the scalar path)."""
    t = torch.zeros(a.size + offset, dtype=torch.float32 if a.dtype == np.float32 else torch.int32, device="cuda")
    v = t[offset:]
    v.copy_(torch.from_numpy(a))
    return v


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


@pytest.mark.parametrize("n", SIZES)
@pytest.mark.parametrize("offset", [0, 1])
def test_blas1_bitexact(cuda, oracle, n, offset):
    a = synth.uniform(1, (n,), -1, 1)
    b = synth.uniform(2, (n,), -1, 1)
    cases = [
        ("fill", lambda x, y: gpu.fill(x, n, 1.25), lambda x, y: oracle.fill(x, 1.25)),
        ("copy", lambda x, y: gpu.copy(n, y, x), lambda x, y: oracle.copy(y, x)),
        ("axpy", lambda x, y: gpu.axpy(n, 2.5, y, x), lambda x, y: oracle.axpy(2.5, y, x)),
        ("scal", lambda x, y: gpu.scal(n, 0.3, x), lambda x, y: oracle.scal(0.3, x)),
        ("mul", lambda x, y: gpu.mul(n, y, x), lambda x, y: oracle.mul(y, x)),
        ("add_scalar", lambda x, y: gpu.addScalar(n, 0.7, x), lambda x, y: oracle.add_scalar(0.7, x)),
        ("constrain", lambda x, y: gpu.constrainArray(n, 0.5, x), lambda x, y: oracle.constrain(0.5, x)),
    ]
    for name, fg, fo in cases:
        x = dev(a, offset)
        y = dev(b, offset)
        fg(x, y)
        want = a.copy()
        fo(want, b.copy())
        assert_bitexact(host(x), want, f"{name} n={n} offset={offset}")


@pytest.mark.parametrize("act", EXACT_ACTS + EXP_ACTS)
@pytest.mark.parametrize("n", [4099, 65536 + 1])
def test_activate_and_gradient(cuda, oracle, act, n):
    a = synth.uniform(3, (n,), -5, 5)
    d = synth.uniform(4, (n,), -1, 1)
    x = dev(a)
    gpu.activateArray(x, n, act)
    y_want = a.copy()
    oracle.activate_array(y_want, act)
    y_got = host(x)
    if act in EXACT_ACTS:
        assert_bitexact(y_got, y_want, f"activate {act}")
    else:
        assert_close(y_got, y_want, f"activate {act}", rtol=1e-5, atol=1e-6)
    # the gradient consumes the activation output; feed both the same y
    dd = dev(d)
    gpu.gradientArray(dev(y_want), n, act, dd)
    g_want = d.copy()
    oracle.gradient_array(y_want, act, g_want)
    assert_bitexact(host(dd), g_want, f"gradient {act}")


BCAST_SHAPES = [(4, 17, 53), (2, 3, 1), (3, 5, 2), (8, 16, 64), (2, 8, 49), (64, 16, 196), (1, 1, 7)]


@pytest.mark.parametrize("shape", BCAST_SHAPES)
def test_broadcast_ops_bitexact(cuda, oracle, shape):
    B, C, S = shape
    n = B * C * S
    x = synth.uniform(5, (n,), -1, 1)
    d = synth.uniform(6, (n,), -1, 1)
    bias = synth.uniform(7, (C,), -1, 1)
    scale = synth.uniform(8, (C,), 0.5, 1.5)
    mean = synth.normal(9, (C,), 0, 0.5)
    var = synth.uniform(10, (C,), 0.5, 2.0)
    md = synth.uniform(11, (C,), -1, 1)
    vd = synth.uniform(12, (C,), -1, 1)

    t = dev(x); gpu.addBias(t, dev(bias), B, C, S)
    w = x.copy(); oracle.add_bias(w, bias, B, C, S)
    assert_bitexact(host(t), w, "add_bias")

    t = dev(x); gpu.scaleBias(t, dev(scale), B, C, S)
    w = x.copy(); oracle.scale_bias(w, scale, B, C, S)
    assert_bitexact(host(t), w, "scale_bias")

    t = dev(x); gpu.normalize(t, dev(mean), dev(var), B, C, S)
    w = x.copy(); oracle.normalize(w, mean, var, B, C, S)
    assert_bitexact(host(t), w, "normalize")

    t = dev(d); gpu.normalizeDelta(dev(x), dev(mean), dev(var), dev(md), dev(vd), B, C, S, t)
    w = d.copy(); oracle.normalize_delta(x, mean, var, md, vd, B, C, S, w)
    assert_bitexact(host(t), w, "normalize_delta")

    for act in (gpu.LEAKY, gpu.RELU, gpu.LINEAR):
        y = torch.empty(n, dtype=torch.float32, device="cuda")
        gpu.bnActForwardInfer(dev(x), y, B, C, S, dev(scale), dev(bias), dev(mean), dev(var), act)
        w = x.copy()
        oracle.normalize(w, mean, var, B, C, S)
        oracle.scale_bias(w, scale, B, C, S)
        oracle.add_bias(w, bias, B, C, S)
        oracle.activate_array(w, act)
        assert_bitexact(host(y), w, f"bn_act_forward_infer act={act}")


MAXPOOL_CASES = [
    (3, 6, 14, 14, 2, 2, 1),   # gputest.zig:393-399
    (2, 3, 13, 13, 3, 2, 2),   # overlapping windows
    (2, 4, 7, 7, 2, 2, 1),     # odd size: last window half outside
    (1, 2, 9, 11, 3, 3, 0),
    (2, 16, 224, 224, 2, 2, 1),  # BASELINE config 2's first pool shape (batch reduced)
    (4, 5, 6, 6, 2, 1, 1),
]


def test_maxpool_2x2_ties_keep_the_first_maximum(cuda, oracle):
    """The vectorised 2x2 / stride-2 path with many equal values: the first maximum in
    (row, col) tap order wins, as in pooling.zig:59-93."""
    B, C, H, W = 2, 4, 8, 16
    x = np.round(synth.uniform(23, (B * C * H * W,), -1, 1) * 2).astype(np.float32) / 2
    oh, ow = H // 2, W // 2
    out = torch.empty(B * C * oh * ow, dtype=torch.float32, device="cuda")
    idx = torch.empty(B * C * oh * ow, dtype=torch.int32, device="cuda")
    gpu.forwardMaxpool(B * C * oh * ow, H, W, C, 2, 2, 1, dev(x), out, idx)
    w_out = np.zeros(B * C * oh * ow, np.float32)
    w_idx = np.zeros(B * C * oh * ow, np.int32)
    oracle.forward_maxpool(B, H, W, C, 2, 2, 1, x, w_out, w_idx)
    assert_bitexact(host(out), w_out, "maxpool values")
    assert (host(idx) == w_idx).all(), "maxpool indices differ"


@pytest.mark.parametrize("case", MAXPOOL_CASES)
def test_maxpool_bitexact(cuda, oracle, case):
    B, C, H, W, size, stride, pad = case
    x = synth.uniform(13, (B * C * H * W,), -1, 1)
    oh = (H + pad - size) // stride + 1
    ow = (W + pad - size) // stride + 1
    out_n = B * C * oh * ow
    out = torch.empty(out_n, dtype=torch.float32, device="cuda")
    idx = torch.empty(out_n, dtype=torch.int32, device="cuda")
    gpu.forwardMaxpool(out_n, H, W, C, stride, size, pad, dev(x), out, idx)
    w_out = np.zeros(out_n, np.float32)
    w_idx = np.zeros(out_n, np.int32)
    oracle.forward_maxpool(B, H, W, C, stride, size, pad, x, w_out, w_idx)
    assert_bitexact(host(out), w_out, "maxpool values")
    assert (host(idx) == w_idx).all(), "maxpool indices differ"
    # backward: scatter-add of the output delta into a non-zero prev_delta
    delta = synth.uniform(14, (out_n,), -1, 1)
    prev0 = synth.uniform(15, (B * C * H * W,), -1, 1)
    prev = dev(prev0)
    gpu.backwardMaxpool(prev0.size, H, W, C, stride, size, pad, dev(delta), prev, idx)
    w_prev = prev0.copy()
    oracle.backward_maxpool(delta, w_idx, w_prev)
    assert_bitexact(host(prev), w_prev, "maxpool backward")


@pytest.mark.parametrize("case", [(3, 6, 14, 14), (256, 1000, 7, 7), (4, 8, 1, 1), (2, 3, 5, 3), (2, 4, 32, 32)])
def test_avgpool(cuda, oracle, case):
    B, C, H, W = case
    S = H * W
    x = synth.normal(16, (B * C * S,), 0, 2)
    out = torch.empty(B * C, dtype=torch.float32, device="cuda")
    gpu.forwardAvgpool(B * C, W, H, C, dev(x), out)
    want = np.zeros(B * C, np.float32)
    oracle.forward_avgpool(B, C, H, W, x, want)
    if S * 4 * 32 <= 96 * 1024:  # planes staged in shared memory: the CPU's summation order
        assert_bitexact(host(out), want, "avgpool")
    else:
        assert_close(host(out), want, "avgpool", rtol=1e-5, atol=1e-6)
    od = synth.uniform(17, (B * C,), -1, 1)
    ind0 = synth.uniform(18, (B * C * S,), -1, 1)
    ind = dev(ind0)
    gpu.backwardAvgpool(B * C, W, H, C, ind, dev(od))
    w = ind0.copy()
    oracle.backward_avgpool(B, C, H, W, od, w)
    assert_bitexact(host(ind), w, "avgpool backward")


@pytest.mark.parametrize("rows,classes", [(8, 137), (256, 1000), (3, 5000), (1, 1), (2, 13001)])
def test_softmax_and_cross_entropy(cuda, oracle, rows, classes):
    n = rows * classes
    x = synth.normal(19, (n,), 0, 2)
    truth = synth.one_hot(20, rows, classes).ravel()
    out = torch.empty(n, dtype=torch.float32, device="cuda")
    gpu.softmax(dev(x), classes, rows, classes, 1, classes, 1, 1.0, out)
    w = np.zeros(n, np.float32)
    oracle.softmax(x, classes, rows, classes, 1, classes, 1, 1.0, w)
    got = host(out)
    assert_close(got, w, "softmax", rtol=1e-5, atol=1e-6)
    delta = torch.empty_like(out)
    err = torch.empty_like(out)
    gpu.softmaxCrossEntropy(n, dev(w), dev(truth), delta, err)
    wd = np.zeros(n, np.float32)
    we = np.zeros(n, np.float32)
    oracle.softmax_cross_entropy(w, truth, wd, we)
    assert_bitexact(host(delta), wd, "xent delta")
    assert_close(host(err), we, "xent err", rtol=1e-5, atol=1e-6)
    # fused softmax + cross entropy + cost
    o2, d2, e2 = (torch.empty_like(out) for _ in range(3))
    cost = torch.zeros(1, dtype=torch.float32, device="cuda")
    gpu.softmaxXent(dev(x), dev(truth), classes, rows, 1.0, o2, d2, e2, cost)
    assert_close(host(o2), w, "fused softmax", rtol=1e-5, atol=1e-6)
    assert_close(host(d2), wd, "fused delta", rtol=1e-5, atol=1e-6)
    assert_close(host(e2), we, "fused err", rtol=1e-5, atol=1e-6)
    want_cost = oracle.sum_array(we)
    assert_close(host(cost), np.array([want_cost], np.float32), "cost")


@pytest.mark.parametrize("temp,stride,groups", [(2.0, 1, 1), (1.0, 1, 3), (1.0, 2, 2), (0.5, 3, 3)])
def test_softmax_strided_groups(cuda, oracle, temp, stride, groups):
    """Grouped and interleaved rows (blas.zig:210-212): with stride s the s groups of a
    batch item interleave (group_offset 1); with stride 1 they are consecutive."""
    batch, n = 4, 50
    batch_offset = n * groups
    size = batch * batch_offset
    x = synth.normal(21, (size,), 0, 1)
    out = dev(np.zeros(size, np.float32))
    group_offset = 1 if stride > 1 else n
    gpu.softmax(dev(x), n, batch, batch_offset, groups, group_offset, stride, temp, out)
    w = np.zeros(size, np.float32)
    oracle.softmax(x, n, batch, batch_offset, groups, group_offset, stride, temp, w)
    assert_close(host(out), w, "strided softmax", rtol=1e-5, atol=1e-6)


@pytest.mark.parametrize("case", [((2, 8, 8, 4), (2, 8, 8, 4), 1.0, 1.0),
                                  ((256, 14, 14, 512), (256, 14, 14, 512), 1.0, 1.0),
                                  ((2, 16, 16, 8), (2, 8, 8, 4), 0.5, 1.5),
                                  ((2, 8, 8, 4), (2, 16, 16, 8), 0.25, 2.0),
                                  ((3, 5, 5, 3), (3, 5, 5, 3), 0.7, 0.3)])
def test_shortcut_bitexact(cuda, oracle, case):
    (b, w1, h1, c1), (_, w2, h2, c2), s1, s2 = case
    add = synth.uniform(22, (b * c1 * h1 * w1,), -1, 1)
    out0 = synth.uniform(23, (b * c2 * h2 * w2,), -1, 1)
    out = dev(out0)
    gpu.shortcut(b, w1, h1, c1, dev(add), w2, h2, c2, s1, s2, out)
    w = out0.copy()
    oracle.shortcut(b, w1, h1, c1, add, w2, h2, c2, s1, s2, w)
    assert_bitexact(host(out), w, "shortcut")


@pytest.mark.parametrize("n", [4099, (1 << 22) + 1])
def test_sgd_momentum_bitexact(cuda, oracle, n):
    w0 = synth.normal(24, (n,), 0, 0.01)
    u0 = synth.normal(25, (n,), 0, 1e-3)
    w = dev(w0)
    u = dev(u0)
    gpu.sgdMomentum(n, w, u, 0.1, 0.9, 5e-4, 128)
    ww, uw = w0.copy(), u0.copy()
    oracle.sgd_update(ww, uw, 0.1, 0.9, 5e-4, 128)
    assert_bitexact(host(w), ww, "sgd weights")
    assert_bitexact(host(u), uw, "sgd weight_updates")


def test_invalid_arguments_raise(cuda):
    x = torch.zeros(8, device="cuda")
    with pytest.raises(gpu.DnbError):
        gpu.activateArray(x, 8, 99)
    with pytest.raises(gpu.DnbError):
        gpu.fill(x, -1, 0.0)
    with pytest.raises(gpu.DnbError):
        gpu.forwardMaxpool(5, 4, 4, 1, 2, 2, 1, x, x, torch.zeros(8, dtype=torch.int32, device="cuda"))
