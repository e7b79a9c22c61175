"""Data-parallel weight update: gradient reduce-scatter, the fused SGD update on this rank's
shard, all-gather of the updated weights.

The reference updates a layer's weights on its one GPU (convolutional.zig:311-335): with
weight_updates accumulated by the backward pass, axpy(-decay*batch, w, wu), axpy(lr/batch,
wu, w), scal(momentum, wu). Across N data-parallel ranks the update must see the sum of every
rank's gradient. Here each rank owns 1/N of the weight vector's update (ZeRO stage 1):

    reduce-scatter (sum) of the ranks' gradients -> this rank's shard of the global gradient
    dnb_axpy(1, gradient shard, momentum shard)     weight_updates += gradient (its shard)
    dnb_sgd_momentum on the shard                   the reference's three ops, one pass
    all-gather of the updated weight shards         every rank holds the same weights

The momentum state (weight_updates) stays sharded: each rank keeps only its 1/N. Every rank
ends with bit-identical weights, since each shard is computed once and broadcast.

ShardedSGD runs the three steps as NCCL collectives around this library's kernels (through a
torch.distributed process group; the same host logic runs over gloo on the CPU in
tests/test_dpsgd_cpu.py with the update supplied by the caller). FusedShardedSGD does all
three in one kernel per rank over NVLink peer memory (dnb_dpsgd_*): each rank reads its
shard's gradients from every rank, updates the shard and stores the new weights into every
rank's weight vector, element by element; the weights and gradients then live in the
library's shared buffers.
"""
from __future__ import annotations


class ShardedSGD:
    """Sharded momentum SGD over `n` replicated weights on `world` ranks."""

    def __init__(self, n: int, world: int, rank: int, dist=None, device=None):
        import torch

        if world > 1 and dist is None:
            raise ValueError("world > 1 needs a torch.distributed module with an initialised process group")
        self.n, self.world, self.rank, self.dist = n, world, rank, dist
        self.shard = -(-n // world)                 # weights per rank (the last shard padded)
        self.n_pad = self.shard * world
        self.lo = rank * self.shard
        self.hi = min(n, self.lo + self.shard)
        dev = device if device is not None else ("cuda" if torch.cuda.is_available() else "cpu")
        # this rank's momentum shard (weight_updates) and the reduced gradient shard
        self.momentum = torch.zeros(self.shard, dtype=torch.float32, device=dev)
        self.grad_shard = torch.empty(self.shard, dtype=torch.float32, device=dev)

    def padded(self, t):
        """A flat view of `t` padded to the collectives' size (a copy only when n is not a
        multiple of the ranks)."""
        import torch

        if t.numel() == self.n_pad:
            return t
        out = torch.zeros(self.n_pad, dtype=t.dtype, device=t.device)
        out[: self.n].copy_(t)
        return out

    def step(self, weights_pad, grads_pad, learning_rate, momentum, decay, batch, update=None):
        """One update. `weights_pad` and `grads_pad` hold n_pad floats (see padded()); the
        gradients are this rank's contribution and are consumed. `update(n, w, wu, lr, mom,
        decay, batch)` is the shard update (default: dnb_axpy + dnb_sgd_momentum on the GPU).
        `batch` is the global batch (the reference's lr/batch and decay*batch scaling)."""
        d = self.dist
        if self.world > 1:
            d.reduce_scatter_tensor(self.grad_shard, grads_pad, op=d.ReduceOp.SUM)
        else:
            self.grad_shard.copy_(grads_pad[: self.shard])
        w_shard = weights_pad[self.rank * self.shard:(self.rank + 1) * self.shard]
        if update is None:
            from . import gpu

            gpu.axpy(self.shard, 1.0, self.grad_shard, self.momentum)
            gpu.sgdMomentum(self.shard, w_shard, self.momentum, learning_rate, momentum, decay, batch)
        else:
            update(self.shard, w_shard, self.momentum, self.grad_shard, learning_rate, momentum, decay, batch)
        if self.world > 1:
            # NCCL gathers in place (the shard is this rank's slice of the output); gloo wants
            # a separate input
            d.all_gather_into_tensor(weights_pad, w_shard if w_shard.is_cuda else w_shard.clone())


class FusedShardedSGD:
    """The same update as ShardedSGD in one kernel per rank over NVLink peer memory. The
    weight vector and the gradient buffer are the library's (`weights`, `grads`: torch
    views of n_pad floats); the host swaps the group's IPC handles once through `dist`."""

    def __init__(self, n: int, world: int, rank: int, dist=None):
        import torch

        from . import gpu

        if world > 1 and dist is None:
            raise ValueError("world > 1 needs a torch.distributed module with an initialised process group")
        self.n, self.world, self.rank = n, world, rank
        self.group, handle, self.weights, self.grads, self.lo, self.shard = gpu.dpsgdInit(rank, world, n)
        handles = [handle]
        if world > 1:
            handles = [None] * world
            dist.all_gather_object(handles, handle)
        gpu.dpsgdConnect(self.group, b"".join(handles))
        self.n_pad = self.shard * world
        self.momentum = torch.zeros(self.shard, dtype=torch.float32, device="cuda")

    def step(self, learning_rate, momentum, decay, batch) -> None:
        from . import gpu

        gpu.dpsgdStep(self.group, self.momentum, learning_rate, momentum, decay, batch)

    def close(self) -> None:
        from . import gpu

        if self.group is not None:
            gpu.dpsgdDestroy(self.group)
            self.group = None
