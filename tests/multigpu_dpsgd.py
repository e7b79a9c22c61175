"""Two-GPU parity of the data-parallel weight update; run as
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29534 tests/multigpu_dpsgd.py
(tests/test_gpu_dpsgd.py::test_two_gpus does so when the box has two GPUs).

Both forms of the update run on the same weights and gradients for two steps: the fused
kernel over NVLink peer memory (dpsgd.FusedShardedSGD) and NCCL reduce-scatter / all-gather
around the library's kernels (dpsgd.ShardedSGD). Every rank's weights must be bit-identical
across ranks, across the two forms, and to the update with the two ranks' gradients summed
(two summands: the order of the sum does not matter); every rank's momentum shard must equal
the NCCL form's."""
from __future__ import annotations

import datetime
import os
import sys

import numpy as np
import torch
import torch.distributed as dist

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(HERE))
sys.path.insert(0, HERE)


def main() -> None:
    rank = int(os.environ["RANK"])
    world = int(os.environ["WORLD_SIZE"])
    local = int(os.environ.get("LOCAL_RANK", rank))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", local))
    from darknet_zig_b200 import gpu
    from darknet_zig_b200.dpsgd import FusedShardedSGD, ShardedSGD
    from parity import assert_bitexact

    gpu.init(local)
    for n in (4099, 1 << 22):
        gw = torch.Generator(device="cuda")
        gw.manual_seed(7)
        w0 = torch.randn(n, generator=gw, device="cuda") * 0.01
        fused = FusedShardedSGD(n, world, rank, dist=dist)
        nccl = ShardedSGD(n, world, rank, dist=dist, device=torch.device("cuda", local))
        fused.weights[:n].copy_(w0)
        w_n = nccl.padded(w0.clone())
        assert fused.shard >= nccl.shard
        for step in range(2):
            gr = torch.Generator(device="cuda")
            gr.manual_seed(100 * step + rank)
            grad = torch.randn(n, generator=gr, device="cuda") * 1e-3
            fused.grads[:n].copy_(grad)
            torch.cuda.synchronize()
            dist.barrier()
            fused.step(0.1, 0.9, 5e-4, 256)
            nccl.step(w_n, nccl.padded(grad), 0.1, 0.9, 5e-4, 256)
            torch.cuda.synchronize()
            gpu.check_device_error()
            wf = fused.weights[:n].cpu().numpy()
            assert_bitexact(wf, w_n[:n].cpu().numpy(), f"fused vs NCCL weights, n={n} step {step}")
            lo = rank * nccl.shard
            k = min(nccl.shard, n - lo)
            # the two forms shard alike when n splits evenly; compare where both own the elements
            if fused.shard == nccl.shard:
                assert_bitexact(fused.momentum[:k].cpu().numpy(), nccl.momentum[:k].cpu().numpy(),
                                f"momentum shard, n={n} step {step}")
            allw = [torch.empty(n, device="cuda") for _ in range(world)]
            dist.all_gather(allw, fused.weights[:n].contiguous())
            for q in range(1, world):
                assert torch.equal(allw[q].view(torch.int32), allw[0].view(torch.int32)), "weights differ between ranks"
        fused.close()
        dist.barrier()
        if rank == 0:
            print(f"multigpu_dpsgd: n={n} x {world} ranks ok", flush=True)
    if rank == 0:
        print("multigpu_dpsgd: ok", flush=True)
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
