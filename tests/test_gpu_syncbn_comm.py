"""The fused sync-BN entry points on one GPU: a one-rank communicator runs the whole
cross-GPU exchange inside the sweep kernel (the CTA owning a channel stores its record
into the rank's buffer and every CTA of the channel waits for its tag) and must give
exactly the single-GPU fused results, call after call (the buffer halves alternate). The
same entries across two GPUs are checked by tests/multigpu_syncbn.py (run under torchrun;
test_two_gpus runs it when the box has two GPUs)."""
from __future__ import annotations

import os
import subprocess
import sys

import numpy as np
import pytest
import torch

from darknet_zig_b200 import _lib, gpu
from parity import assert_bitexact
from test_gpu_bn import dev, host, make_inputs

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("shape", [(8, 16, 64), (16, 40, 196), (128, 128, 1024), (128, 256, 784), (16, 40, 169)])
def test_one_rank_communicator_matches_the_fused_kernels(cuda, shape, monkeypatch):
    # sync-BN never takes the single-GPU small-channel kernel: compare like with like
    monkeypatch.setenv("DNB_BN_SMALL", "0")
    B, C, S = shape
    comm, handle = gpu.commInit(0, 1, C)
    try:
        gpu.commConnect(comm, handle)
        for rep in range(3):  # three calls each way: both buffer halves, tags 1..6
            x, gamma, beta, delta, rm0, rv0 = make_inputs(shape, seed=20 + rep)
            outs = []
            for fused in (False, True):
                y = torch.empty(x.size, dtype=torch.float32, device="cuda")
                xn = torch.empty_like(y)
                mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
                rm, rv = dev(rm0), dev(rv0)
                dx = torch.empty_like(y)
                bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(4))
                if fused:
                    gpu.syncbnActForwardTrain(comm, dev(x), y, xn, B, C, S, dev(gamma), dev(beta), mean, var, rm, rv,
                                              gpu.LEAKY)
                    gpu.syncbnActBackward(comm, dev(x), None, dev(delta), dx, B, C, S, dev(gamma), dev(beta), mean,
                                          var, bu, su, md, vd, gpu.LEAKY)
                else:
                    gpu.bnActForwardTrain(dev(x), y, xn, B, C, S, dev(gamma), dev(beta), mean, var, rm, rv,
                                          gpu.LEAKY)
                    gpu.bnActBackward(dev(x), None, dev(delta), dx, B, C, S, dev(gamma), dev(beta), mean, var, bu,
                                      su, md, vd, gpu.LEAKY)
                outs.append([host(t) for t in (y, xn, mean, var, rm, rv, dx, bu, su, md, vd)])
            gpu.check_device_error()
            names = ("y", "x_norm", "mean", "var", "rolling_mean", "rolling_var", "dx", "bias_updates",
                     "scale_updates", "mean_delta", "variance_delta")
            for n, a, b in zip(names, outs[0], outs[1]):
                assert_bitexact(b, a, f"{n} (call {rep})")
    finally:
        gpu.commDestroy(comm)


def test_unsupported_shape_is_reported(cuda):
    B, C, S = 3, 5, 9  # spatial % 4 != 0 and an element count that is not a multiple of 4
    comm, handle = gpu.commInit(0, 1, C)
    try:
        gpu.commConnect(comm, handle)
        x = torch.randn(B * C * S, device="cuda")
        y = torch.empty_like(x)
        z = [torch.zeros(C, device="cuda") for _ in range(6)]
        with pytest.raises(_lib.DnbError) as e:
            gpu.syncbnActForwardTrain(comm, x, y, None, B, C, S, *z, gpu.LEAKY)
        assert e.value.status == 5
    finally:
        gpu.commDestroy(comm)


def test_two_gpus():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs (runs in the multi-GPU calls)")
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node", "2", "--master-addr",
           "127.0.0.1", "--master-port", "29533", os.path.join(root, "tests", "multigpu_syncbn.py")]
    # NVLS off: a rank of the timeout case leaves no collective in flight, but no NVLink
    # multicast object should be involved in a failure test either
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, capture_output=True, text=True, timeout=900, env=env)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "multigpu_syncbn: ok" in r.stdout
