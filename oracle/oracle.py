"""TEST INFRASTRUCTURE -- Python bindings of the CPU oracle.

`Oracle` wraps oracle/_build/liboracle.so (the C restatement of the reference's CPU ops,
ref_ops.c) and `RefEmulation` wraps oracle/_ref/libref_emulate.so (the reference's own
kernel file run on the host). Both work in place on numpy float32 / int32 arrays, with
the argument order of the reference functions they restate. `RefGpu` wraps
oracle/_ref/libref_gpu.so, the same kernel file built for the B200 (device pointers).

Only tests/, __graft_entry__.smoke() and bench.py's baseline legs (the CPU baseline and the
reference arm) use this module; the product never imports it.
"""
from __future__ import annotations

import ctypes as C
import os

import numpy as np

from . import build_oracle as _b

_f32p = C.POINTER(C.c_float)
_i32p = C.POINTER(C.c_int32)
_i64 = C.c_int64


def _fp(a):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags.c_contiguous, (a.dtype, a.flags)
    return a.ctypes.data_as(_f32p)


def _ip(a):
    assert a.dtype == np.int32 and a.flags.c_contiguous
    return a.ctypes.data_as(_i32p)


class Oracle:
    """The C restatement of blas.zig / activations.zig / pooling.zig / layer sequences."""

    def __init__(self, path: str | None = None):
        path = path or _b.build_oracle()
        self.lib = C.CDLL(path)
        L = self.lib
        L.ref_activate.restype = C.c_float
        L.ref_activate.argtypes = [C.c_float, C.c_int]
        L.ref_gradient.restype = C.c_float
        L.ref_gradient.argtypes = [C.c_float, C.c_int]
        L.ref_sum_array.restype = C.c_float
        L.ref_sum_array.argtypes = [_f32p, _i64]
        L.ref_maxpool_out_dim.restype = _i64
        L.ref_maxpool_out_dim.argtypes = [_i64] * 4
        L.oracle_get_threads.restype = C.c_int

    # threading (CPU baseline only; results are identical for any thread count)
    def set_threads(self, n: int) -> None:
        self.lib.oracle_set_threads(C.c_int(n))

    def threads(self) -> int:
        return self.lib.oracle_get_threads()

    # blas.zig:13-46
    def fill(self, x, alpha):
        self.lib.ref_fill(_fp(x), _i64(x.size), C.c_float(alpha))

    def copy(self, src, dst):
        self.lib.ref_copy(_fp(src), _fp(dst), _i64(src.size))

    def axpy(self, alpha, x, y):
        self.lib.ref_axpy(C.c_float(alpha), _fp(x), _fp(y), _i64(x.size))

    def scal(self, alpha, x):
        self.lib.ref_scal(C.c_float(alpha), _fp(x), _i64(x.size))

    def mul(self, x, y):
        self.lib.ref_mul(_fp(x), _fp(y), _i64(x.size))

    def add_scalar(self, alpha, x):
        self.lib.ref_add_scalar(C.c_float(alpha), _fp(x), _i64(x.size))

    def constrain(self, alpha, x):
        self.lib.ref_constrain(C.c_float(alpha), _fp(x), _i64(x.size))

    # activations.zig
    def activate(self, x: float, act: int) -> float:
        return self.lib.ref_activate(C.c_float(x), C.c_int(act))

    def gradient(self, y: float, act: int) -> float:
        return self.lib.ref_gradient(C.c_float(y), C.c_int(act))

    def activate_array(self, x, act):
        self.lib.ref_activate_array(_fp(x), _i64(x.size), C.c_int(act))

    def gradient_array(self, y, act, delta):
        self.lib.ref_gradient_array(_fp(y), _i64(y.size), C.c_int(act), _fp(delta))

    # blas.zig:53-100
    def add_bias(self, out, biases, batch, filters, spatial):
        self.lib.ref_add_bias(_fp(out), _fp(biases), _i64(batch), _i64(filters), _i64(spatial))

    def scale_bias(self, out, scales, batch, filters, spatial):
        self.lib.ref_scale_bias(_fp(out), _fp(scales), _i64(batch), _i64(filters), _i64(spatial))

    def backward_bias(self, bias_updates, delta, batch, filters, spatial):
        self.lib.ref_backward_bias(_fp(bias_updates), _fp(delta), _i64(batch), _i64(filters), _i64(spatial))

    def backward_scale(self, x_norm, delta, batch, filters, spatial, scale_updates):
        self.lib.ref_backward_scale(_fp(x_norm), _fp(delta), _i64(batch), _i64(filters), _i64(spatial),
                                    _fp(scale_updates))

    # blas.zig:106-204
    def mean(self, x, batch, filters, spatial, out):
        self.lib.ref_mean(_fp(x), _i64(batch), _i64(filters), _i64(spatial), _fp(out))

    def variance(self, x, mean, batch, filters, spatial, out):
        self.lib.ref_variance(_fp(x), _fp(mean), _i64(batch), _i64(filters), _i64(spatial), _fp(out))

    def normalize(self, x, mean, variance, batch, filters, spatial):
        self.lib.ref_normalize(_fp(x), _fp(mean), _fp(variance), _i64(batch), _i64(filters), _i64(spatial))

    def mean_delta(self, delta, variance, batch, filters, spatial, out):
        self.lib.ref_mean_delta(_fp(delta), _fp(variance), _i64(batch), _i64(filters), _i64(spatial), _fp(out))

    def variance_delta(self, x, delta, mean, variance, batch, filters, spatial, out):
        self.lib.ref_variance_delta(_fp(x), _fp(delta), _fp(mean), _fp(variance), _i64(batch), _i64(filters),
                                    _i64(spatial), _fp(out))

    def normalize_delta(self, x, mean, variance, mean_delta, variance_delta, batch, filters, spatial, delta):
        self.lib.ref_normalize_delta(_fp(x), _fp(mean), _fp(variance), _fp(mean_delta), _fp(variance_delta),
                                     _i64(batch), _i64(filters), _i64(spatial), _fp(delta))

    # blas.zig:213-252, utils.zig:71-75
    def softmax(self, inp, n, batch, batch_offset, groups, group_offset, stride, temp, out):
        self.lib.ref_softmax(_fp(inp), _i64(n), _i64(batch), _i64(batch_offset), _i64(groups), _i64(group_offset),
                             _i64(stride), C.c_float(temp), _fp(out))

    def softmax_cross_entropy(self, pred, truth, delta, err):
        self.lib.ref_softmax_cross_entropy(_fp(pred), _fp(truth), _fp(delta), _fp(err), _i64(pred.size))

    def sum_array(self, a) -> float:
        return self.lib.ref_sum_array(_fp(a), _i64(a.size))

    # blas.zig:290-322
    def shortcut(self, batch, w1, h1, c1, add, w2, h2, c2, s1, s2, out):
        self.lib.ref_shortcut(_i64(batch), _i64(w1), _i64(h1), _i64(c1), _fp(add), _i64(w2), _i64(h2), _i64(c2),
                              C.c_float(s1), C.c_float(s2), _fp(out))

    # pooling.zig
    def maxpool_out_dim(self, n, size, stride, pad) -> int:
        return self.lib.ref_maxpool_out_dim(n, size, stride, pad)

    def forward_maxpool(self, batch, in_h, in_w, in_c, stride, size, pad, inp, out, indexes):
        self.lib.ref_forward_maxpool(_i64(batch), _i64(in_h), _i64(in_w), _i64(in_c), _i64(stride), _i64(size),
                                     _i64(pad), _fp(inp), _fp(out), _ip(indexes))

    def backward_maxpool(self, delta, indexes, prev_delta):
        self.lib.ref_backward_maxpool(_i64(delta.size), _fp(delta), _ip(indexes), _fp(prev_delta))

    def forward_avgpool(self, batch, c, h, w, inp, out):
        self.lib.ref_forward_avgpool(_i64(batch), _i64(c), _i64(h), _i64(w), _fp(inp), _fp(out))

    def backward_avgpool(self, batch, c, h, w, out_delta, in_delta):
        self.lib.ref_backward_avgpool(_i64(batch), _i64(c), _i64(h), _i64(w), _fp(out_delta), _fp(in_delta))

    # layer sequences
    def bn_forward_layer(self, x, y, x_saved, x_norm, batch, filters, spatial, scales, biases, mean, variance,
                         rolling_mean, rolling_variance, train, act):
        self.lib.ref_bn_forward_layer(_fp(x), _fp(y), _fp(x_saved), _fp(x_norm), _i64(batch), _i64(filters),
                                      _i64(spatial), _fp(scales), _fp(biases), _fp(mean), _fp(variance),
                                      _fp(rolling_mean), _fp(rolling_variance), C.c_int(int(train)), C.c_int(act))

    def bn_backward_layer(self, x, x_norm, y, delta, batch, filters, spatial, scales, mean, variance, bias_updates,
                          scale_updates, mean_delta, variance_delta, act):
        self.lib.ref_bn_backward_layer(_fp(x), _fp(x_norm), _fp(y), _fp(delta), _i64(batch), _i64(filters),
                                       _i64(spatial), _fp(scales), _fp(mean), _fp(variance), _fp(bias_updates),
                                       _fp(scale_updates), _fp(mean_delta), _fp(variance_delta), C.c_int(act))

    def sgd_update(self, w, wu, learning_rate, momentum, decay, batch):
        self.lib.ref_sgd_update(_fp(w), _fp(wu), _i64(w.size), C.c_float(learning_rate), C.c_float(momentum),
                                C.c_float(decay), _i64(batch))


class RefEmulation:
    """The reference's darknet_kernels.hip run on the host (argument order of gpu.zig)."""

    def __init__(self, path: str | None = None):
        path = path or _b.build_ref_emulation()
        if path is None or not os.path.exists(path):
            raise FileNotFoundError("reference emulation library not built (reference tree absent)")
        self.lib = C.CDLL(path)

    def __getattr__(self, name):
        return getattr(self.lib, "ref_emu_" + name)


class RefGpu:
    """The reference's darknet_kernels.hip built for sm_100a (oracle/_ref/libref_gpu.so),
    launched with the reference's own grids. Arguments are device pointers (ints, e.g. a
    torch tensor's data_ptr()) and a cudaStream_t handle; sizes are the reference's c_int.
    Used by the GPU tests as a second parity anchor and by bench.py's reference arm as the
    per-op GPU baseline."""

    _P = C.c_void_p

    def __init__(self, path: str | None = None):
        path = path or _b.build_ref_gpu()
        if path is None or not os.path.exists(path):
            raise FileNotFoundError("reference GPU kernel library not built (reference tree absent)")
        self.lib = C.CDLL(path)
        P, I, F = self._P, C.c_int, C.c_float
        L = self.lib
        L.ref_gpu_conv_bn_forward.argtypes = [P] * 9 + [I, I, I, I, P]
        L.ref_gpu_conv_bn_backward.argtypes = [P] * 11 + [I, I, I, I, P]
        L.ref_gpu_sgd_weights.argtypes = [I, F, F, F, I, P, P, P]
        for f in (L.ref_gpu_conv_bn_forward, L.ref_gpu_conv_bn_backward, L.ref_gpu_sgd_weights):
            f.restype = C.c_int
        self.launches_forward = L.ref_gpu_launches_forward()
        self.launches_backward = L.ref_gpu_launches_backward()
        self.launches_sgd = L.ref_gpu_launches_sgd()

    def _call(self, name: str, *args) -> None:
        # ctypes converts surplus arguments by guesswork (a pointer passed as a C int is
        # truncated), so the count is checked against the declared argtypes first
        fn = getattr(self.lib, "ref_gpu_" + name)
        if len(args) != len(fn.argtypes):
            raise TypeError(f"ref_gpu_{name} takes {len(fn.argtypes)} arguments, {len(args)} given")
        rc = fn(*args)
        if rc != 0:
            raise RuntimeError(f"reference kernels ({name}): cudaError {rc}")

    def conv_bn_forward(self, output, x, x_norm, mean, variance, rolling_mean, rolling_variance, scales, biases,
                        batch, filters, spatial, act, stream=0):
        """convolutional.zig:263-268 + batchnorm.zig:129-153 (train): `output` in place."""
        self._call("conv_bn_forward", output, x, x_norm, mean, variance, rolling_mean, rolling_variance, scales,
                   biases, batch, filters, spatial, act, stream)

    def conv_bn_backward(self, output, delta, x, x_norm, mean, variance, scales, bias_updates, scale_updates,
                         mean_delta, variance_delta, batch, filters, spatial, act, stream=0):
        """convolutional.zig:279-282 + batchnorm.zig:155-170: `delta` in place."""
        self._call("conv_bn_backward", output, delta, x, x_norm, mean, variance, scales, bias_updates,
                   scale_updates, mean_delta, variance_delta, batch, filters, spatial, act, stream)

    def sgd_weights(self, nweights, learning_rate, momentum, decay, batch, weights, weight_updates, stream=0):
        """convolutional.zig:332-334."""
        self._call("sgd_weights", nweights, learning_rate, momentum, decay, batch, weights, weight_updates, stream)


_ORACLE: Oracle | None = None


def get_oracle() -> Oracle:
    global _ORACLE
    if _ORACLE is None:
        _ORACLE = Oracle()
    return _ORACLE
