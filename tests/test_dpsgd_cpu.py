"""The data-parallel weight update's host logic on the CPU: two gloo ranks run
dpsgd.ShardedSGD (reduce-scatter of the gradients, the shard update, all-gather of the
weights) with the shard update done by the CPU restatement of the reference's SGD
(convolutional.zig:330-334). After two steps every rank must hold weights bit-identical to
one process updating the whole vector with the summed gradient, and its momentum shard must
equal that process's weight_updates on the shard. The weight count is odd, so the last shard
is padded. Nothing here touches a GPU."""
from __future__ import annotations

import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

N_W, LR, MOM, DECAY, BATCH = 1001, 0.1, 0.9, 5e-4, 256


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _grads(rank, step):
    return np.random.default_rng(100 * step + rank).standard_normal(N_W).astype(np.float32) * 1e-2


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from darknet_zig_b200.dpsgd import ShardedSGD
        from oracle.oracle import get_oracle

        orc = get_oracle()

        def update(n, w, wu, g, lr, mom, decay, batch):
            wn, wun = w.numpy(), wu.numpy()
            orc.axpy(1.0, g.numpy(), wun)  # weight_updates += gradient
            orc.sgd_update(wn, wun, lr, mom, decay, batch)

        opt = ShardedSGD(N_W, world, rank, dist=dist, device="cpu")
        w0 = np.random.default_rng(7).standard_normal(N_W).astype(np.float32)
        w = opt.padded(torch.from_numpy(w0.copy()))
        for step in range(2):
            g = opt.padded(torch.from_numpy(_grads(rank, step)))
            opt.step(w, g, LR, MOM, DECAY, BATCH, update=update)
        out[rank] = (w[:N_W].numpy().copy(), opt.momentum.numpy().copy(), opt.lo, opt.hi)
    finally:
        dist.destroy_process_group()


def test_two_ranks_match_one_process():
    from oracle.oracle import get_oracle

    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(out)
    orc = get_oracle()
    w = np.random.default_rng(7).standard_normal(N_W).astype(np.float32)
    wu = np.zeros(N_W, np.float32)
    for step in range(2):
        g = _grads(0, step) + _grads(1, step)  # two ranks: the sum's order does not matter
        orc.axpy(1.0, g, wu)
        orc.sgd_update(w, wu, LR, MOM, DECAY, BATCH)
    for r in range(2):
        wr, mr, lo, hi = res[r]
        assert np.array_equal(wr.view(np.uint32), w.view(np.uint32)), f"rank {r} weights"
        assert np.array_equal(mr[: hi - lo].view(np.uint32), wu[lo:hi].view(np.uint32)), f"rank {r} momentum"
