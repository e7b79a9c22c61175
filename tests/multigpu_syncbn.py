"""Two-GPU parity of the fused sync-BN entries; run as
    python -m torch.distributed.run --nnodes=1 --nproc-per-node 2 --master-addr 127.0.0.1 \\
        --master-port 29533 tests/multigpu_syncbn.py
(tests/test_gpu_syncbn_comm.py::test_two_gpus does so when the box has two GPUs).

Each rank holds its own batch shard; the forward and backward run through
syncbn.SyncBN (the communicator path: records exchanged inside the kernel over NVLink), once
with the default kernel choice (the L2 sweep where it takes the shape) and once with the
cluster-per-channel kernel. Rank 0 gathers every rank's tensors and checks the whole batch
against the CPU oracle with the same bars as the single-GPU tests: statistics within
tolerance of the whole batch's, identical on every rank; y, rolling statistics and dx
bit-identical to the reference op sequence given the kernel's own per-channel values; the
backward sums within tolerance.

Then a rank that never makes its fused call: with a 200 ms wait limit, rank 1 skips one
forward. Rank 0's kernel must give up after the limit and report DNB_ERR_TIMEOUT through
dnb_check_device_error (which clears the error word and abort flag); both ranks then
recreate their communicators and a fresh step must pass the oracle check again. The failure
is made on the host (a skipped call); nothing faults a GPU, and NVLS is off."""
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

    gpu.init(local)
    act = gpu.LEAKY
    paths = {"default": {}, "cluster": {"DNB_BN_SWEEP": "0"}}
    cases = [(p, sh) for p in paths for sh in [(8, 16, 64), (16, 40, 196), (16, 40, 169), (128, 128, 1024)]]
    cases.append(("default", (128, 256, 784)))
    for path, shape in cases:
        for k in ("DNB_BN_SWEEP",):
            os.environ.pop(k, None)
        os.environ.update(paths[path])
        check_step(rank, world, path, shape, act)
    for path in paths:
        os.environ.pop("DNB_BN_SWEEP", None)
        os.environ.update(paths[path])
        check_skipped_call(rank, world, path, act)
    os.environ.pop("DNB_BN_SWEEP", None)
    if rank == 0:
        print("multigpu_syncbn: ok", flush=True)
    dist.destroy_process_group()


def check_step(rank, world, path, shape, act) -> None:
    from darknet_zig_b200 import gpu, synth, syncbn
    from parity import assert_bitexact, assert_close, exact_channel_sum
    from test_gpu_bn import check_forward_stats, oracle_backward_given_stats, oracle_bn_apply

    B, C, S = shape
    x = synth.normal(900 + rank, (B * C * S,), 0.25, 1.0)
    delta = synth.normal(950 + rank, (B * C * S,), 0.0, 1.0)
    gamma = synth.uniform(101, (C,), 0.5, 1.5)
    beta = synth.normal(102, (C,), 0.0, 0.1)
    rm0 = synth.normal(104, (C,), 0.0, 0.5)
    rv0 = synth.uniform(105, (C,), 0.5, 2.0)
    d = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    layer = syncbn.SyncBN(B, C, S, world=world, dist=dist, rank=rank)
    assert layer.comm is not None
    xd, dd = d(x), d(delta)
    y = torch.empty_like(xd)
    mean, var = torch.zeros(C, device="cuda"), torch.zeros(C, device="cuda")
    rm, rv = d(rm0), d(rv0)
    layer.forward(xd, y, d(gamma), d(beta), mean, var, rm, rv, act)
    dx = torch.empty_like(xd)
    bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(4))
    layer.backward(xd, dd, dx, d(gamma), d(beta), mean, var, bu, su, md, vd, act)
    torch.cuda.synchronize()
    gpu.check_device_error()
    layer.close()

    def gather(t):
        out = [torch.empty_like(t) for _ in range(world)]
        dist.all_gather(out, t.contiguous())
        return [o.cpu().numpy() for o in out]

    xs, ys, ds, dxs = gather(xd), gather(y), gather(dd), gather(dx)
    per_rank = [gather(t) for t in (mean, var, rm, rv, bu, su, md, vd)]
    if rank == 0:
        from oracle.oracle import get_oracle

        orc = get_oracle()
        for vals in per_rank:  # identical on every rank
            for r in range(1, world):
                assert_bitexact(vals[r], vals[0], "rank-identical per-channel output")
        m, v, rm_g, rv_g, bu_g, su_g, md_g, vd_g = (vals[0] for vals in per_rank)
        whole = (B * world, C, S)
        x_all, y_all, d_all, dx_all = (np.concatenate(a) for a in (xs, ys, ds, dxs))
        check_forward_stats(orc, x_all.copy(), whole, m, v)
        rm_w, rv_w = rm0.copy(), rv0.copy()
        orc.scal(0.99, rm_w)
        orc.axpy(np.float32(1) - np.float32(0.99), m, rm_w)
        orc.scal(0.99, rv_w)
        orc.axpy(np.float32(1) - np.float32(0.99), v, rv_w)
        assert_bitexact(rm_g, rm_w, "rolling_mean")
        assert_bitexact(rv_g, rv_w, "rolling_variance")
        _, y_w = oracle_bn_apply(orc, x_all, m, v, gamma, beta, whole, act)
        assert_bitexact(y_all, y_w, "y")
        g, gs, dx_w = oracle_backward_given_stats(orc, x_all, y_all, d_all, whole, gamma, m, v, md_g, vd_g, act)
        assert_bitexact(dx_all, dx_w, "dx")
        Bw = B * world
        s1, s1n = exact_channel_sum(g, Bw, C, S)
        assert_close(bu_g, s1, "bias_updates", atol=1e-6, scale=s1n)
        xn = x_all.copy()
        orc.normalize(xn, m, v, Bw, C, S)
        s2, s2n = exact_channel_sum(g * xn, Bw, C, S)
        assert_close(su_g, s2, "scale_updates", atol=1e-6, scale=s2n)
        inv = (-1.0 / np.sqrt(v.astype(np.float32) + np.float32(1e-5))).astype(np.float64)
        sgs, sgsn = exact_channel_sum(gs, Bw, C, S)
        assert_close(md_g, sgs * inv, "mean_delta", atol=1e-6, scale=sgsn * np.abs(inv))
        print(f"multigpu_syncbn: {path} shape {shape} x {world} ranks ok", flush=True)
    dist.barrier()


def check_skipped_call(rank, world, path, act) -> None:
    from darknet_zig_b200 import _lib, gpu, synth, syncbn

    B, C, S = 8, 16, 64
    x = torch.from_numpy(synth.normal(700 + rank, (B * C * S,), 0.0, 1.0)).cuda()
    y = torch.empty_like(x)
    g, b = torch.ones(C, device="cuda"), torch.zeros(C, device="cuda")
    m, v, rm, rv = (torch.zeros(C, device="cuda") for _ in range(4))
    gpu.set_wait_limit_ms(200)
    try:
        layer = syncbn.SyncBN(B, C, S, world=world, dist=dist, rank=rank)
        layer.forward(x, y, g, b, m, v, rm, rv, act)  # call 1 on both ranks
        torch.cuda.synchronize()
        gpu.check_device_error()
        dist.barrier()
        if rank == 0:
            layer.forward(x, y, g, b, m, v, rm, rv, act)  # call 2: rank 1 never joins it
            torch.cuda.synchronize()
            try:
                gpu.check_device_error()
                raise AssertionError("the lone rank's kernel did not report its timeout")
            except _lib.DnbError as e:
                assert e.status == 3, e
            gpu.check_device_error()  # the error word and the abort flag were cleared
        dist.barrier()
        layer.close()
        # fresh communicators on every rank, and a step that must be right again
        layer = syncbn.SyncBN(B, C, S, world=world, dist=dist, rank=rank)
        layer.forward(x, y, g, b, m, v, rm, rv, act)
        torch.cuda.synchronize()
        gpu.check_device_error()
        layer.close()
    finally:
        gpu.set_wait_limit_ms(2000)
    check_step(rank, world, path, (8, 16, 64), act)
    if rank == 0:
        print(f"multigpu_syncbn: {path} a skipped call timed out and the ranks recovered", flush=True)
    dist.barrier()


if __name__ == "__main__":
    main()
