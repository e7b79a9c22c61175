"""Sync-BN: batchnorm + activation whose per-channel statistics span every rank's shard.

The reference has no multi-GPU path (README.md:313-317); this is the data-parallel form of
its batchnorm layer (batchnorm.zig:129-174) for BASELINE config 4. One process per GPU;
each rank holds batch/world images.

  world == 1: the fused single-GPU kernels (dnb_bn_act_forward_train / _backward).
  world  > 1, fused (default): dnb_syncbn_act_forward_train / _backward on a communicator
              (dnb_comm_*): one kernel per direction that exchanges the per-channel records
              with the other GPUs itself, over NVLink peer memory, while it streams; the host
              only swaps the communicator's IPC handles once (here through the process group).
  world  > 1, split (shapes the fused kernel does not take, or fused=False): the split
              entry points around two small collectives per layer step:
    forward   dnb_syncbn_forward_partials -> all_gather of [C,2] fp64 (mean, M2) per rank
              -> dnb_syncbn_forward_apply (Chan merge of the ranks' records, then apply)
    backward  dnb_syncbn_backward_partials -> all_reduce(SUM) of [C,2] fp64 (sum g,
              sum g*(x-mean)) -> dnb_syncbn_backward_apply
The split path's collectives go through a torch.distributed process group (NCCL on GPUs;
the same exchange functions run over gloo on the CPU in tests/test_syncbn_cpu.py).

`combine_forward_partials` is the host restatement of the merge the device performs
(k_fwd_finalize), used to check the protocol without a GPU.
"""
from __future__ import annotations

import numpy as np

from . import gpu
from ._lib import call


def combine_forward_partials(gathered: np.ndarray, count_per_rank: int):
    """[R, C, 2] (mean_r, M2_r) records of equal-count shards -> (mean, unbiased var), fp64
    (Chan et al.'s pairwise update, all ranks at once)."""
    g = np.asarray(gathered, np.float64)
    mu = g[:, :, 0].mean(axis=0)
    m2 = (g[:, :, 1] + count_per_rank * (g[:, :, 0] - mu[None, :]) ** 2).sum(axis=0)
    n = count_per_rank * g.shape[0]
    return mu, m2 / (n - 1)


def local_forward_partials(x: np.ndarray, batch: int, filters: int, spatial: int) -> np.ndarray:
    """Host form of dnb_syncbn_forward_partials: [C, 2] (mean, M2) of this shard, fp64."""
    v = x.reshape(batch, filters, spatial).transpose(1, 0, 2).reshape(filters, -1).astype(np.float64)
    m = v.mean(axis=1)
    return np.stack([m, ((v - m[:, None]) ** 2).sum(axis=1)], axis=1)


def local_backward_partials(g: np.ndarray, x: np.ndarray, mean: np.ndarray, batch: int, filters: int,
                            spatial: int) -> np.ndarray:
    """Host form of dnb_syncbn_backward_partials given the activation-gradient terms
    g = delta * act'(y): [C, 2] (sum g, sum g * (x - mean)) of this shard, fp64."""
    gv = g.reshape(batch, filters, spatial).transpose(1, 0, 2).reshape(filters, -1).astype(np.float64)
    xv = x.reshape(batch, filters, spatial).transpose(1, 0, 2).reshape(filters, -1).astype(np.float64)
    return np.stack([gv.sum(axis=1), (gv * (xv - np.asarray(mean, np.float64)[:, None])).sum(axis=1)], axis=1)


def gather_forward_partials(dist, part, gathered) -> None:
    """The forward exchange: every rank's [C, 2] fp64 (mean, M2) record into
    gathered[world, C, 2], in rank order (so every rank merges identically)."""
    if hasattr(dist, "all_gather_into_tensor") and part.is_cuda:
        dist.all_gather_into_tensor(gathered, part)
    else:
        dist.all_gather(list(gathered.unbind(0)), part)


def reduce_backward_partials(dist, part) -> None:
    """The backward exchange: [C, 2] fp64 (sum g, sum g*(x-mean)) summed over ranks, in place."""
    dist.all_reduce(part)


class SyncBN:
    def __init__(self, batch: int, filters: int, spatial: int, world: int = 1, dist=None, fused: bool = True,
                 rank: int = 0):
        self.batch, self.filters, self.spatial = batch, filters, spatial
        self.world = world
        self.dist = dist
        if world > 1 and dist is None:
            raise ValueError("world > 1 needs a torch.distributed module with an initialised process group")
        self._bufs = None
        self.comm = None
        if world > 1 and fused:
            # every rank's IPC handle, swapped once through the process group
            self.comm, handle = gpu.commInit(rank, world, filters)
            handles = [None] * world
            dist.all_gather_object(handles, handle)
            gpu.commConnect(self.comm, b"".join(handles))

    def close(self) -> None:
        if self.comm is not None:
            gpu.commDestroy(self.comm)
            self.comm = None

    def _buffers(self, device):
        import torch

        if self._bufs is None:
            C = self.filters
            self._bufs = {
                "fpart": torch.empty(C, 2, dtype=torch.float64, device=device),
                "gathered": torch.empty(self.world, C, 2, dtype=torch.float64, device=device),
                "bpart": torch.empty(C, 2, dtype=torch.float64, device=device),
            }
        return self._bufs

    def forward(self, x, y, gamma, beta, mean, var, rolling_mean, rolling_variance, act, x_norm=None):
        B, C, S = self.batch, self.filters, self.spatial
        if self.world == 1:
            gpu.bnActForwardTrain(x, y, x_norm, B, C, S, gamma, beta, mean, var, rolling_mean, rolling_variance, act)
            return
        if self.comm is not None:
            gpu.syncbnActForwardTrain(self.comm, x, y, x_norm, B, C, S, gamma, beta, mean, var, rolling_mean,
                                      rolling_variance, act)
            return
        b = self._buffers(x.device)
        s = gpu._s()
        call("syncbn_forward_partials", gpu._p(x), B, C, S, b["fpart"].data_ptr(), s)
        gather_forward_partials(self.dist, b["fpart"], b["gathered"])
        call("syncbn_forward_apply", gpu._p(x), gpu._p(y), gpu._p(x_norm), B, C, S, b["gathered"].data_ptr(),
             self.world, gpu._p(gamma), gpu._p(beta), gpu._p(mean), gpu._p(var), gpu._p(rolling_mean),
             gpu._p(rolling_variance), int(act), s)

    def backward(self, x, delta, dx, gamma, beta, mean, var, bias_updates, scale_updates, mean_delta,
                 variance_delta, act, y=None):
        B, C, S = self.batch, self.filters, self.spatial
        if self.world == 1:
            gpu.bnActBackward(x, y, delta, dx, B, C, S, gamma, beta, mean, var, bias_updates, scale_updates,
                              mean_delta, variance_delta, act)
            return
        if self.comm is not None:
            gpu.syncbnActBackward(self.comm, x, y, delta, dx, B, C, S, gamma, beta, mean, var, bias_updates,
                                  scale_updates, mean_delta, variance_delta, act)
            return
        b = self._buffers(x.device)
        s = gpu._s()
        call("syncbn_backward_partials", gpu._p(x), gpu._p(y), gpu._p(delta), B, C, S, gpu._p(gamma), gpu._p(beta),
             gpu._p(mean), gpu._p(var), int(act), b["bpart"].data_ptr(), s)
        reduce_backward_partials(self.dist, b["bpart"])
        call("syncbn_backward_apply", gpu._p(x), gpu._p(y), gpu._p(delta), gpu._p(dx), B, C, S, B * S * self.world,
             b["bpart"].data_ptr(), gpu._p(gamma), gpu._p(beta), gpu._p(mean), gpu._p(var), gpu._p(bias_updates),
             gpu._p(scale_updates), gpu._p(mean_delta), gpu._p(variance_delta), int(act), s)
