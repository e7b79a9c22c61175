"""Layer-level callers of the ops, mirroring the reference's GPU layer bodies.

`BatchNorm` holds the batch-normalisation state a convolutional layer carries
(layer.zig:145-278: scales, biases, mean, variance, rolling stats, updates, x, x_norm) and
runs either
  * the fused path: one dnb_bn_act_forward_train / dnb_bn_act_backward launch, or
  * the reference's own op sequence (batchnorm.zig:129-174 with the activation of
    convolutional.zig:269/280), one gpu.* op per reference launch,
so the two can be compared on the device. `sgd_update` is convolutional.updateGpu
(convolutional.zig:311-335) and `softmax_forward` is misc.forwardSoftmaxGpu
(misc.zig:59-72).
"""
from __future__ import annotations

import torch

from . import gpu

ROLLING_MOMENTUM = 0.99  # batchnorm.zig:16


class BatchNorm:
    def __init__(self, batch: int, filters: int, h: int, w: int, activation: int = gpu.LEAKY, device="cuda"):
        self.batch, self.filters, self.h, self.w = batch, filters, h, w
        self.spatial = h * w
        self.n = batch * filters * self.spatial
        self.activation = activation
        z = lambda: torch.zeros(filters, dtype=torch.float32, device=device)  # noqa: E731
        self.scales = torch.ones(filters, dtype=torch.float32, device=device)  # batchnorm.zig:40
        self.biases = z()
        self.scale_updates, self.bias_updates = z(), z()
        self.mean, self.variance = z(), z()
        self.rolling_mean, self.rolling_variance = z(), z()
        self.mean_delta, self.variance_delta = z(), z()
        self.x = None       # the pre-BN conv output kept for the backward (l.x)
        self.x_norm = None  # l.x_norm (reference path, or fused with keep_x_norm)
        self.output = None  # l.output (activated)

    # -- forward ------------------------------------------------------------------------
    def forward(self, x: torch.Tensor, train: bool = True, fused: bool = True, keep_x_norm: bool = False):
        """x: the conv output [batch, filters, h, w]; returns the activated output."""
        B, C, S = self.batch, self.filters, self.spatial
        if fused:
            self.x = x
            self.output = torch.empty_like(x)
            if train:
                self.x_norm = torch.empty_like(x) if keep_x_norm else None
                gpu.bnActForwardTrain(x, self.output, self.x_norm, B, C, S, self.scales, self.biases, self.mean,
                                      self.variance, self.rolling_mean, self.rolling_variance, self.activation)
            else:
                gpu.bnActForwardInfer(x, self.output, B, C, S, self.scales, self.biases, self.rolling_mean,
                                      self.rolling_variance, self.activation)
            return self.output
        # batchnorm.zig:129-152 (conv layer: l.output already holds the conv result)
        out = x.clone()
        self.x = torch.empty_like(x)
        gpu.copy(self.n, out, self.x)
        if train:
            gpu.mean(out, B, C, S, self.mean)
            gpu.variance(out, self.mean, B, C, S, self.variance)
            gpu.scal(C, ROLLING_MOMENTUM, self.rolling_mean)
            gpu.axpy(C, 1 - ROLLING_MOMENTUM, self.mean, self.rolling_mean)
            gpu.scal(C, ROLLING_MOMENTUM, self.rolling_variance)
            gpu.axpy(C, 1 - ROLLING_MOMENTUM, self.variance, self.rolling_variance)
            gpu.normalize(out, self.mean, self.variance, B, C, S)
            self.x_norm = torch.empty_like(x)
            gpu.copy(self.n, out, self.x_norm)
        else:
            gpu.normalize(out, self.rolling_mean, self.rolling_variance, B, C, S)
        gpu.scaleBias(out, self.scales, B, C, S)
        gpu.addBias(out, self.biases, B, C, S)
        gpu.activateArray(out, self.n, self.activation)  # convolutional.zig:269
        self.output = out
        return out

    # -- backward -----------------------------------------------------------------------
    def backward(self, delta: torch.Tensor, train: bool = True, fused: bool = True, use_output: bool = False):
        """delta: dL/d(output); overwritten with dL/dx (as l.delta is), and returned."""
        B, C, S = self.batch, self.filters, self.spatial
        mean_in = self.mean if train else self.rolling_mean  # batchnorm.zig:159-160
        var_in = self.variance if train else self.rolling_variance
        if fused:
            gpu.bnActBackward(self.x, self.output if use_output else None, delta, delta, B, C, S, self.scales,
                              self.biases, mean_in, var_in, self.bias_updates, self.scale_updates, self.mean_delta,
                              self.variance_delta, self.activation)
            return delta
        gpu.gradientArray(self.output, self.n, self.activation, delta)  # convolutional.zig:280
        gpu.backwardBias(self.bias_updates, delta, B, C, S)
        gpu.backwardScale(self.x_norm, delta, B, C, S, self.scale_updates)
        gpu.scaleBias(delta, self.scales, B, C, S)
        gpu.meanDelta(delta, var_in, B, C, S, self.mean_delta)
        gpu.varianceDelta(self.x, delta, mean_in, var_in, B, C, S, self.variance_delta)
        gpu.normalizeDelta(self.x, mean_in, var_in, self.mean_delta, self.variance_delta, B, C, S, delta)
        return delta


def sgd_update(weights, weight_updates, biases, bias_updates, scales, scale_updates, learning_rate: float,
               momentum: float, decay: float, batch: int, fused: bool = True) -> None:
    """convolutional.updateGpu (convolutional.zig:311-335), SGD branch."""
    b = float(batch)
    n = biases.numel()
    gpu.axpy(n, learning_rate / b, bias_updates, biases)
    gpu.scal(n, momentum, bias_updates)
    if scales is not None:
        gpu.axpy(n, learning_rate / b, scale_updates, scales)
        gpu.scal(n, momentum, scale_updates)
    nw = weights.numel()
    if fused:
        gpu.sgdMomentum(nw, weights, weight_updates, learning_rate, momentum, decay, batch)
    else:
        gpu.axpy(nw, -decay * b, weights, weight_updates)
        gpu.axpy(nw, learning_rate / b, weight_updates, weights)
        gpu.scal(nw, momentum, weight_updates)


def softmax_forward(inp, truth, batch: int, inputs: int, temperature: float = 1.0, fused: bool = True):
    """misc.forwardSoftmaxGpu (misc.zig:59-72) for groups = 1. Returns
    (output, delta, loss, cost) with cost a 1-element device tensor."""
    out = torch.empty_like(inp)
    delta = torch.empty_like(inp)
    loss = torch.empty_like(inp)
    cost = torch.empty(1, dtype=torch.float32, device=inp.device)
    if fused:
        gpu.softmaxXent(inp, truth, inputs, batch, temperature, out, delta, loss, cost)
    else:
        gpu.softmax(inp, inputs, batch, inputs, 1, inputs, 1, temperature, out)
        gpu.softmaxCrossEntropy(batch * inputs, out, truth, delta, loss)
        cost.copy_(loss.sum().reshape(1))
    return out, delta, loss, cost
