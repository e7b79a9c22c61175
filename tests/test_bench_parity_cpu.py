"""bench.py's pre-timing parity check, run on the CPU over two gloo ranks.

Each rank builds a shard and the results a correct sync-BN step produces on it (global
statistics over both shards, y and dx from the per-channel values with one float32 rounding
per operation, SGD with single-rounding fused multiply-adds), then calls
`check_step_parity` as bench.py does. A correct step must pass on both ranks; a single
flipped bit in one rank's y, or statistics that differ between ranks, must fail on both
(the verdict is all-reduced). Nothing here touches a GPU."""
from __future__ import annotations

import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)

import bench  # noqa: E402

f32 = np.float32


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _step_results(rank, world, B, C, S, NW, plant):
    rng = np.random.default_rng(10 + rank)
    x = rng.standard_normal(B * C * S).astype(f32)
    delta = rng.standard_normal(B * C * S).astype(f32)
    grng = np.random.default_rng(3)
    gamma = (grng.random(C) + 0.5).astype(f32)
    beta = (grng.standard_normal(C) * 0.1).astype(f32)
    rm0 = (grng.standard_normal(C) * 0.5).astype(f32)
    rv0 = (grng.random(C) * 1.5 + 0.5).astype(f32)
    # global statistics over every rank's shard (each rank regenerates the others' data)
    shards = [np.random.default_rng(10 + r).standard_normal(B * C * S).astype(f32).reshape(B, C, S)
              for r in range(world)]
    allx = np.concatenate(shards, axis=0).transpose(1, 0, 2).reshape(C, -1).astype(np.float64)
    n = allx.shape[1]
    mean = allx.mean(axis=1).astype(f32)
    var = (((allx - allx.mean(axis=1, keepdims=True)) ** 2).sum(axis=1) / (n - 1)).astype(f32)
    if plant == "stats" and rank == 1:
        var = var.copy()
        var[0] = np.nextafter(var[0], f32(np.inf))
    rm = np.array([bench.fma_f32(f32(1) - f32(0.99), mean[c], rm0[c] * f32(0.99)) for c in range(C)], f32)
    rv = np.array([bench.fma_f32(f32(1) - f32(0.99), var[c], rv0[c] * f32(0.99)) for c in range(C)], f32)
    xs = x.reshape(B, C, S)
    mc = mean[None, :, None]
    inv = (f32(1) / (np.sqrt(var) + f32(0.000001)))[None, :, None]
    y = bench.leaky_f32((xs - mc) * inv * gamma[None, :, None] + beta[None, :, None])
    gr = delta.reshape(B, C, S) * np.where(y > f32(0), f32(1), f32(0.1))
    # backward sums over both shards (float64), then the reference's per-channel closing
    s1 = np.zeros(C)
    s2 = np.zeros(C)
    for r in range(world):
        xr = shards[r]
        dr = np.random.default_rng(10 + r)
        dr.standard_normal(B * C * S)
        dlt = dr.standard_normal(B * C * S).astype(f32).reshape(B, C, S)
        yr = bench.leaky_f32((xr - mc) * inv * gamma[None, :, None] + beta[None, :, None])
        gg = (dlt * np.where(yr > f32(0), f32(1), f32(0.1))).astype(np.float64)
        s1 += gg.sum(axis=(0, 2))
        s2 += (gg * (xr.astype(np.float64) - mc.astype(np.float64))).sum(axis=(0, 2))
    bu = s1.astype(f32)
    su = (s2 * inv.ravel().astype(np.float64)).astype(f32)
    md = (f32(-1.0) * s1.astype(f32) / np.sqrt(var + f32(0.00001))).astype(f32)
    vd = (s2.astype(f32) * f32(-0.5) * np.power(var + f32(0.00001), f32(-1.5))).astype(f32)
    denom = f32(n)
    inv2 = (f32(1) / np.sqrt(var + f32(0.00001)))[None, :, None]
    dx = (gr * gamma[None, :, None]) * inv2 + (vd[None, :, None] * f32(2) * (xs - mc)) / denom + (md / denom)[None, :, None]
    if plant == "y" and rank == 1:
        y = y.copy()
        y.reshape(-1)[5] = np.nextafter(y.reshape(-1)[5], f32(np.inf))
    # SGD on the replicated weights
    wr = np.random.default_rng(99)
    w0 = (wr.standard_normal(NW) * 0.01).astype(f32)
    wu0 = (wr.standard_normal(NW) * 1e-3).astype(f32)
    b32 = f32(B * world)
    a_decay = f32(-f32(bench.SGD_DECAY) * b32)
    a_lr = f32(f32(bench.SGD_LR) / b32)
    w = np.empty_like(w0)
    wu = np.empty_like(wu0)
    for i in range(NW):
        u1 = bench.fma_f32(a_decay, w0[i], wu0[i])
        w[i] = bench.fma_f32(a_lr, u1, w0[i])
        wu[i] = f32(u1 * f32(bench.SGD_MOMENTUM))
    T = torch.from_numpy
    return dict(x=T(x), delta=T(delta), y=T(y.reshape(-1)), dx=T(dx.reshape(-1).astype(f32)), gamma=T(gamma),
                beta=T(beta), mean=T(mean), var=T(var), rm0=rm0, rv0=rv0, rm=T(rm), rv=T(rv), bu=T(bu), su=T(su),
                md=T(md), vd=T(vd), w0=w0, wu0=wu0, w=T(w), wu=T(wu))


def _rank(rank, world, port, plant, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        B, C, S, NW = 3, 4, 10, 2048
        r = _step_results(rank, world, B, C, S, NW, plant)
        # the checker samples 2048 weights with its own seed: with NW == 2048 it takes them all
        idx = np.sort(np.random.default_rng(7).choice(NW, size=2048, replace=False))
        ok, detail = bench.check_step_parity(dist, world, B, C, S, r["x"], r["delta"], r["y"], r["dx"], r["gamma"],
                                             r["beta"], r["mean"], r["var"], r["rm0"], r["rv0"], r["rm"], r["rv"],
                                             r["bu"], r["su"], r["md"], r["vd"], r["w0"][idx], r["wu0"][idx], r["w"],
                                             r["wu"], B * world)
        out[rank] = (ok, detail.get("rank_failures", []))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("plant", ["none", "y", "stats"])
def test_two_ranks(plant):
    ctx = mp.get_context("spawn")
    with ctx.Manager() as m:
        out = m.dict()
        port = _free_port()
        procs = [ctx.Process(target=_rank, args=(r, 2, port, plant, out)) for r in range(2)]
        for p in procs:
            p.start()
        for p in procs:
            p.join(timeout=240)
        assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
        res = dict(out)
    if plant == "none":
        assert res[0][0] and res[1][0], res
    else:
        assert not res[0][0] and not res[1][0], res
        assert res[1][1], res  # rank 1 names what failed
        if plant == "y":
            assert any(s.startswith("y:") for s in res[1][1]), res


def test_round_f32_ties_to_even():
    from fractions import Fraction

    one = Fraction(1)
    ulp = Fraction(2) ** -23
    assert bench.round_f32(one + ulp / 2) == f32(1.0)          # tie: 1.0 has the even mantissa
    assert bench.round_f32(one + 3 * ulp / 2) == f32(1.0) + f32(2.0 ** -22)  # tie: up to even
    assert bench.fma_f32(f32(0.1), f32(3.0), f32(-0.3)) == np.float32(np.float64(f32(0.1)) * 3.0 - np.float64(f32(0.3)))
