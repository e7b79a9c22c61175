"""The fused data-parallel weight update (dnb_dpsgd_*) on the GPU.

One rank: a group of one must give exactly dnb_axpy(1, g, wu) followed by dnb_sgd_momentum,
step after step (the kernel's arithmetic is theirs). Two ranks (when the box has two GPUs):
tests/multigpu_dpsgd.py under torchrun checks the fused kernel against the NCCL form
(dpsgd.ShardedSGD) and against the update with the gradients summed in rank order, bit for
bit, on every rank."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from darknet_zig_b200 import gpu
from darknet_zig_b200.dpsgd import FusedShardedSGD
from parity import assert_bitexact

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("n", [1, 4099, 1 << 20])
def test_one_rank_matches_axpy_then_sgd(cuda, n):
    opt = FusedShardedSGD(n, 1, 0)
    try:
        g = torch.Generator(device="cuda")
        g.manual_seed(n)
        w0 = torch.randn(n, generator=g, device="cuda") * 0.01
        opt.weights[:n].copy_(w0)
        w_ref = w0.clone()
        wu_ref = torch.zeros(opt.shard, device="cuda")
        for step in range(2):
            grad = torch.randn(n, generator=g, device="cuda") * 1e-3
            opt.grads[:n].copy_(grad)
            opt.step(0.1, 0.9, 5e-4, 256)
            gpad = torch.zeros(opt.shard, device="cuda")
            gpad[:n] = grad
            gpu.axpy(opt.shard, 1.0, gpad, wu_ref)
            gpu.sgdMomentum(n, w_ref, wu_ref[:n], 0.1, 0.9, 5e-4, 256)
            torch.cuda.synchronize()
            gpu.check_device_error()
            assert_bitexact(opt.weights[:n].cpu().numpy(), w_ref.cpu().numpy(), f"weights after step {step}")
            assert_bitexact(opt.momentum[:n].cpu().numpy(), wu_ref[:n].cpu().numpy(), f"momentum after step {step}")
    finally:
        opt.close()


def test_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (runs in the multi-GPU calls)")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29534", os.path.join(root, "tests", "multigpu_dpsgd.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "multigpu_dpsgd: ok" in r.stdout
