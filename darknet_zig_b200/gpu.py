"""The reference's GPU array-op layer (src/gpu.zig:483-830), re-exposed over libdnb200.

Each function keeps the name, argument order and meaning of the gpu.zig wrapper it
replaces; buffers are torch CUDA tensors (the reference's non-owning Buf{ptr,len},
gpu.zig:117-134) and every op runs on torch's current stream. Where the reference panics
on a failed launch (gpu.zig:48-55,443-449) these raise DnbError. Fused entries that have
no gpu.zig counterpart follow after the mirrored ones.
"""
from __future__ import annotations

import torch

from ._lib import DnbError, call, lib  # noqa: F401  (DnbError re-exported)

# activations.zig:11-27
LOGISTIC, RELU, RELIE, LINEAR, RAMP, TANH, PLSE, LEAKY, ELU, LOGGY, STAIR, HARDTAN, LHTAN, SELU = range(14)
ACTIVATIONS = {
    "logistic": LOGISTIC, "relu": RELU, "relie": RELIE, "linear": LINEAR, "ramp": RAMP, "tanh": TANH,
    "plse": PLSE, "leaky": LEAKY, "elu": ELU, "loggy": LOGGY, "stair": STAIR, "hardtan": HARDTAN,
    "lhtan": LHTAN, "selu": SELU,
}


def _p(t, dtype=torch.float32):
    """Device pointer of a CUDA tensor (None -> NULL)."""
    if t is None:
        return None
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise TypeError("expected a CUDA tensor")
    if t.dtype != dtype or not t.is_contiguous():
        raise TypeError(f"expected a contiguous {dtype} tensor, got {t.dtype}")
    return t.data_ptr()


def _s():
    return torch.cuda.current_stream().cuda_stream


# ---- device / memory (gpu.zig:259-410) --------------------------------------------------

def init(device: int = 0) -> None:
    call("init", device)


def set_sync_after_launch(on: bool) -> None:
    """DARKNET_GPU_SYNC (gpu.zig:173-183): synchronise and check after every op."""
    call("set_sync_after_launch", int(bool(on)))


def check_device_error() -> None:
    """Raises DnbError(DNB_ERR_TIMEOUT) if a device-side wait gave up since the last check."""
    call("check_device_error")


def set_wait_limit_ms(ms: int) -> None:
    call("set_wait_limit_ms", int(ms))


def launch_count() -> int:
    """Device-side launches (kernels and memsets) the library has issued in this process."""
    import ctypes

    n = ctypes.c_ulonglong(0)
    call("launch_count", ctypes.byref(n))
    return int(n.value)


def sync() -> None:
    call("sync")


def alloc(n: int, device=None) -> torch.Tensor:
    """gpu.alloc (gpu.zig:362-369): n zero-filled floats."""
    return torch.zeros(int(n), dtype=torch.float32, device=device or "cuda")


def allocInts(n: int, device=None) -> torch.Tensor:  # noqa: N802 (gpu.zig:373)
    return torch.zeros(int(n), dtype=torch.int32, device=device or "cuda")


def make(host) -> torch.Tensor:
    """gpu.make (gpu.zig:378-382): a device copy of a host array."""
    return torch.as_tensor(host, dtype=torch.float32).contiguous().cuda()


def pull(b: torch.Tensor):
    """gpu.pull (gpu.zig:395-399): the buffer's contents on the host (numpy)."""
    return b.detach().cpu().numpy()


# ---- elementwise (gpu.zig:483-521) ------------------------------------------------------

def fill(x, n, alpha):
    call("fill", _p(x), int(n), float(alpha), _s())


def copy(n, x, y):
    call("copy", int(n), _p(x), _p(y), _s())


def axpy(n, alpha, x, y):
    call("axpy", int(n), float(alpha), _p(x), _p(y), _s())


def scal(n, alpha, x):
    call("scal", int(n), float(alpha), _p(x), _s())


def mul(n, x, y):
    call("mul", int(n), _p(x), _p(y), _s())


def addScalar(n, alpha, x):  # noqa: N802
    call("add_scalar", int(n), float(alpha), _p(x), _s())


def constrainArray(n, alpha, x):  # noqa: N802
    call("constrain", int(n), float(alpha), _p(x), _s())


def activateArray(x, n, a):  # noqa: N802
    call("activate_array", _p(x), int(n), int(a), _s())


def gradientArray(x, n, a, delta):  # noqa: N802
    call("gradient_array", _p(x), int(n), int(a), _p(delta), _s())


# ---- bias / scale (gpu.zig:527-555) -----------------------------------------------------

def addBias(output, biases, batch, filters, spatial):  # noqa: N802
    call("add_bias", _p(output), _p(biases), int(batch), int(filters), int(spatial), _s())


def scaleBias(output, scales, batch, filters, spatial):  # noqa: N802
    call("scale_bias", _p(output), _p(scales), int(batch), int(filters), int(spatial), _s())


def backwardBias(bias_updates, delta, batch, filters, spatial):  # noqa: N802
    call("backward_bias", _p(bias_updates), _p(delta), int(batch), int(filters), int(spatial), _s())


def backwardScale(x_norm, delta, batch, filters, spatial, scale_updates):  # noqa: N802
    call("backward_scale", _p(x_norm), _p(delta), int(batch), int(filters), int(spatial), _p(scale_updates), _s())


# ---- batch normalisation (gpu.zig:561-612) ----------------------------------------------

def mean(x, batch, filters, spatial, out):
    call("mean", _p(x), int(batch), int(filters), int(spatial), _p(out), _s())


def variance(x, mean_in, batch, filters, spatial, out):
    call("variance", _p(x), _p(mean_in), int(batch), int(filters), int(spatial), _p(out), _s())


def normalize(x, mean_in, variance_in, batch, filters, spatial):
    call("normalize", _p(x), _p(mean_in), _p(variance_in), int(batch), int(filters), int(spatial), _s())


def meanDelta(delta, variance_in, batch, filters, spatial, out):  # noqa: N802
    call("mean_delta", _p(delta), _p(variance_in), int(batch), int(filters), int(spatial), _p(out), _s())


def varianceDelta(x, delta, mean_in, variance_in, batch, filters, spatial, out):  # noqa: N802
    call("variance_delta", _p(x), _p(delta), _p(mean_in), _p(variance_in), int(batch), int(filters), int(spatial),
         _p(out), _s())


def normalizeDelta(x, mean_in, variance_in, mean_delta_in, variance_delta_in, batch, filters, spatial,  # noqa: N802
                   delta):
    call("normalize_delta", _p(x), _p(mean_in), _p(variance_in), _p(mean_delta_in), _p(variance_delta_in),
         int(batch), int(filters), int(spatial), _p(delta), _s())


# ---- softmax and losses (gpu.zig:614-633) -----------------------------------------------

def softmax(input, n, batch, batch_offset, groups, group_offset, stride, temp, output):  # noqa: A002
    call("softmax", _p(input), int(n), int(batch), int(batch_offset), int(groups), int(group_offset), int(stride),
         float(temp), _p(output), _s())


def softmaxCrossEntropy(n, pred, truth, delta, err):  # noqa: N802
    call("softmax_cross_entropy", int(n), _p(pred), _p(truth), _p(delta), _p(err), _s())


# ---- pooling, shortcut (gpu.zig:725-802) ------------------------------------------------

def forwardMaxpool(out_n, in_h, in_w, in_c, stride, size, pad, input, output, indexes):  # noqa: N802,A002
    call("forward_maxpool", int(out_n), int(in_h), int(in_w), int(in_c), int(stride), int(size), int(pad),
         _p(input), _p(output), _p(indexes, torch.int32), _s())


def backwardMaxpool(in_n, in_h, in_w, in_c, stride, size, pad, delta, prev_delta, indexes):  # noqa: N802
    call("backward_maxpool", int(in_n), int(in_h), int(in_w), int(in_c), int(stride), int(size), int(pad),
         _p(delta), _p(prev_delta), _p(indexes, torch.int32), _s())


def forwardAvgpool(n, w, h, c, input, output):  # noqa: N802,A002
    call("forward_avgpool", int(n), int(w), int(h), int(c), _p(input), _p(output), _s())


def backwardAvgpool(n, w, h, c, in_delta, out_delta):  # noqa: N802
    call("backward_avgpool", int(n), int(w), int(h), int(c), _p(in_delta), _p(out_delta), _s())


def shortcut(batch, w1, h1, c1, add, w2, h2, c2, s1, s2, out):
    call("shortcut", int(batch), int(w1), int(h1), int(c1), _p(add), int(w2), int(h2), int(c2), float(s1),
         float(s2), _p(out), _s())


# ---- fused entries ------------------------------------------------------------------------

def bnActForwardTrain(x, y, x_norm, batch, filters, spatial, scales, biases, mean_out, variance_out,  # noqa: N802
                      rolling_mean, rolling_variance, act):
    call("bn_act_forward_train", _p(x), _p(y), _p(x_norm), int(batch), int(filters), int(spatial), _p(scales),
         _p(biases), _p(mean_out), _p(variance_out), _p(rolling_mean), _p(rolling_variance), int(act), _s())


def bnActForwardInfer(x, y, batch, filters, spatial, scales, biases, rolling_mean, rolling_variance,  # noqa: N802
                      act):
    call("bn_act_forward_infer", _p(x), _p(y), int(batch), int(filters), int(spatial), _p(scales), _p(biases),
         _p(rolling_mean), _p(rolling_variance), int(act), _s())


def bnActForwardFromStats(x, y, x_norm, batch, filters, spatial, pieces, npieces, scales, biases, mean,  # noqa: N802
                          variance, rolling_mean, rolling_variance, act):
    """Training forward from the producer's per-piece (count, mean, M2) statistics, fp64
    [npieces][filters][3]; no counterpart in gpu.zig."""
    call("bn_act_forward_from_stats", _p(x), _p(y), _p(x_norm), int(batch), int(filters), int(spatial),
         _p(pieces, torch.float64),
         int(npieces), _p(scales), _p(biases), _p(mean), _p(variance), _p(rolling_mean), _p(rolling_variance),
         int(act), _s())


def bnActBackward(x, y, delta, dx, batch, filters, spatial, scales, biases, mean_in, variance_in,  # noqa: N802
                  bias_updates, scale_updates, mean_delta_out, variance_delta_out, act):
    call("bn_act_backward", _p(x), _p(y), _p(delta), _p(dx), int(batch), int(filters), int(spatial), _p(scales),
         _p(biases), _p(mean_in), _p(variance_in), _p(bias_updates), _p(scale_updates), _p(mean_delta_out),
         _p(variance_delta_out), int(act), _s())


def sgdMomentum(n, weights, weight_updates, learning_rate, momentum, decay, batch):  # noqa: N802
    call("sgd_momentum", int(n), _p(weights), _p(weight_updates), float(learning_rate), float(momentum),
         float(decay), int(batch), _s())


def softmaxXent(input, truth, n, batch, temp, output, delta, err, cost=None):  # noqa: N802,A002
    call("softmax_xent", _p(input), _p(truth), int(n), int(batch), float(temp), _p(output), _p(delta), _p(err),
         _p(cost), _s())


# ---- fused sync-BN across GPUs (no reference counterpart) --------------------------------

def commInit(rank: int, world: int, max_channels: int):  # noqa: N802
    """A sync-BN communicator on the current device: (handle, this rank's 64-byte IPC handle)."""
    import ctypes

    comm = ctypes.c_void_p(0)
    ipc = ctypes.create_string_buffer(64)
    call("comm_init", int(rank), int(world), int(max_channels), ipc, ctypes.byref(comm))
    return comm.value, ipc.raw


def commConnect(comm, handles: bytes) -> None:  # noqa: N802
    """Opens the peers' exchange buffers; handles = every rank's 64-byte IPC handle, rank order."""
    import ctypes

    call("comm_connect", ctypes.c_void_p(comm), ctypes.create_string_buffer(bytes(handles), len(handles)))


def commDestroy(comm) -> None:  # noqa: N802
    import ctypes

    call("comm_destroy", ctypes.c_void_p(comm))


def syncbnActForwardTrain(comm, x, y, x_norm, batch, filters, spatial, scales, biases, mean_out,  # noqa: N802
                          variance_out, rolling_mean, rolling_variance, act):
    import ctypes

    call("syncbn_act_forward_train", ctypes.c_void_p(comm), _p(x), _p(y), _p(x_norm), int(batch), int(filters),
         int(spatial), _p(scales), _p(biases), _p(mean_out), _p(variance_out), _p(rolling_mean),
         _p(rolling_variance), int(act), _s())


def syncbnActBackward(comm, x, y, delta, dx, batch, filters, spatial, scales, biases, mean_in,  # noqa: N802
                      variance_in, bias_updates, scale_updates, mean_delta_out, variance_delta_out, act):
    import ctypes

    call("syncbn_act_backward", ctypes.c_void_p(comm), _p(x), _p(y), _p(delta), _p(dx), int(batch), int(filters),
         int(spatial), _p(scales), _p(biases), _p(mean_in), _p(variance_in), _p(bias_updates), _p(scale_updates),
         _p(mean_delta_out), _p(variance_delta_out), int(act), _s())



# ---- data-parallel weight update over NVLink (no reference counterpart) -----------------

class _DeviceArray:
    """A float32 device vector owned by the library, seen by torch through
    __cuda_array_interface__ (no copy)."""

    def __init__(self, ptr: int, n: int):
        self.__cuda_array_interface__ = {"shape": (int(n),), "typestr": "<f4", "data": (int(ptr), False),
                                         "version": 3, "strides": None}


def dpsgdInit(rank: int, world: int, n: int):  # noqa: N802
    """A data-parallel update group on the current device: (group, 64-byte IPC handle,
    weights, gradients, shard_lo, shard_n); weights and gradients are torch views of the
    library's shared vectors (padded length world * shard_n)."""
    import ctypes

    group = ctypes.c_void_p(0)
    ipc = ctypes.create_string_buffer(64)
    w, g = ctypes.c_void_p(0), ctypes.c_void_p(0)
    lo, sn = ctypes.c_int64(0), ctypes.c_int64(0)
    call("dpsgd_init", int(rank), int(world), int(n), ipc, ctypes.byref(w), ctypes.byref(g), ctypes.byref(lo),
         ctypes.byref(sn), ctypes.byref(group))
    n_pad = sn.value * world
    wt = torch.as_tensor(_DeviceArray(w.value, n_pad), device="cuda")
    gt = torch.as_tensor(_DeviceArray(g.value, n_pad), device="cuda")
    return group.value, ipc.raw, wt, gt, lo.value, sn.value


def dpsgdConnect(group, handles: bytes) -> None:  # noqa: N802
    import ctypes

    call("dpsgd_connect", ctypes.c_void_p(group), ctypes.create_string_buffer(bytes(handles), len(handles)))


def dpsgdStep(group, momentum, learning_rate, momentum_coef, decay, batch) -> None:  # noqa: N802
    import ctypes

    call("dpsgd_step", ctypes.c_void_p(group), _p(momentum), float(learning_rate), float(momentum_coef),
         float(decay), int(batch), _s())


def dpsgdDestroy(group) -> None:  # noqa: N802
    import ctypes

    call("dpsgd_destroy", ctypes.c_void_p(group))
