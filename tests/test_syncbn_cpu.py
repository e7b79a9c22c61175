"""Sync-BN's exchange protocol on the CPU: two gloo ranks, no GPU.

Each rank reduces its own batch shard to per-channel records with the host forms of the
split entry points (syncbn.local_forward_partials / local_backward_partials), exchanges
them with the same functions SyncBN uses over NCCL (gather_forward_partials,
reduce_backward_partials), and merges. The merged statistics must be identical on both
ranks and agree with the reference's mean / unbiased variance (blas.zig:106-135) of the
whole batch. Failures are made on the host: a rank that raises before the exchange, and a
rank that stays alive but never joins it; the surviving rank must get an error from the
process group within its timeout instead of waiting for good. A rank that joins late but
within the timeout delays the exchange without changing its result."""
from __future__ import annotations

import json
import multiprocessing as mp
import os
import socket
import time

import numpy as np
import pytest

from parity import assert_close

B, C, S = 3, 5, 12  # per-rank shard: batch, channels, spatial
WORLD = 2
PG_TIMEOUT_S = 5


def _free_port() -> int:
    with socket.socket() as sk:
        sk.bind(("127.0.0.1", 0))
        return sk.getsockname()[1]


def _shard(rank: int):
    from darknet_zig_b200 import synth

    x = synth.normal(700 + rank, (B * C * S,), 0.3, 1.2)
    g = synth.normal(800 + rank, (B * C * S,), 0.0, 1.0)
    return x, g


def _worker(rank: int, port: int, mode: str, outdir: str) -> None:
    import datetime

    import torch
    import torch.distributed as dist

    from darknet_zig_b200 import syncbn

    res: dict = {"rank": rank}
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=WORLD,
                            timeout=datetime.timedelta(seconds=PG_TIMEOUT_S))
    t0 = time.monotonic()
    try:
        x, g = _shard(rank)
        part = torch.from_numpy(syncbn.local_forward_partials(x, B, C, S))
        gathered = torch.empty(WORLD, C, 2, dtype=torch.float64)
        if mode == "raise" and rank == 1:
            raise RuntimeError("injected failure before the exchange")
        if mode == "delay" and rank == 1:
            time.sleep(PG_TIMEOUT_S / 2)  # late, but within the process group's timeout
        if mode == "absent" and rank == 1:
            time.sleep(PG_TIMEOUT_S + 4)  # alive, but never joins the exchange
            res["absent"] = True
        else:
            syncbn.gather_forward_partials(dist, part, gathered)
            mu, var = syncbn.combine_forward_partials(gathered.numpy(), B * S)
            bpart = torch.from_numpy(syncbn.local_backward_partials(g, x, mu.astype(np.float32), B, C, S))
            syncbn.reduce_backward_partials(dist, bpart)
            res.update(mean=mu.tolist(), var=var.tolist(), bsum=bpart.numpy().tolist())
    except Exception as e:  # recorded for the parent to check
        res["error"] = f"{type(e).__name__}: {str(e)[:300]}"
    res["seconds"] = time.monotonic() - t0
    with open(os.path.join(outdir, f"rank{rank}.json"), "w") as f:
        json.dump(res, f)
    try:
        dist.destroy_process_group()
    except Exception:
        pass


def _run(mode: str, tmp_path) -> list[dict]:
    ctx = mp.get_context("spawn")
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, port, mode, str(tmp_path))) for r in range(WORLD)]
    for p in procs:
        p.start()
    deadline = time.monotonic() + 120
    for p in procs:
        p.join(max(1.0, deadline - time.monotonic()))
    for p in procs:
        if p.is_alive():  # our own child: kill it by its pid
            p.kill()
            p.join()
            pytest.fail(f"rank process {p.pid} did not finish ({mode})")
    out = []
    for r in range(WORLD):
        with open(tmp_path / f"rank{r}.json") as f:
            out.append(json.load(f))
    return out


def test_forward_and_backward_exchange_match_the_whole_batch(oracle, tmp_path):
    res = _run("ok", tmp_path)
    for r in res:
        assert "error" not in r, r
    # identical on every rank
    assert res[0]["mean"] == res[1]["mean"] and res[0]["var"] == res[1]["var"]
    assert res[0]["bsum"] == res[1]["bsum"]
    # the reference's statistics of the concatenated batch (batch is the outer dimension)
    xs, gs = zip(*(_shard(r) for r in range(WORLD)))
    x_all = np.concatenate(xs)
    g_all = np.concatenate(gs)
    m_ref = np.zeros(C, np.float32)
    v_ref = np.zeros(C, np.float32)
    oracle.mean(x_all.copy(), B * WORLD, C, S, m_ref)
    oracle.variance(x_all.copy(), m_ref, B * WORLD, C, S, v_ref)
    assert_close(np.float32(res[0]["mean"]), m_ref, "sync-BN mean")
    assert_close(np.float32(res[0]["var"]), v_ref, "sync-BN variance")
    # backward sums against float64 sums over the whole batch
    mu = np.asarray(res[0]["mean"], np.float32)
    xv = x_all.reshape(B * WORLD, C, S).astype(np.float64)
    gv = g_all.reshape(B * WORLD, C, S).astype(np.float64)
    s1 = gv.sum(axis=(0, 2))
    s2 = (gv * (xv - mu.astype(np.float64)[None, :, None])).sum(axis=(0, 2))
    got = np.asarray(res[0]["bsum"])
    np.testing.assert_allclose(got[:, 0], s1, rtol=1e-12, atol=1e-12)
    np.testing.assert_allclose(got[:, 1], s2, rtol=1e-12, atol=1e-12)


def test_a_rank_that_raises_ends_the_exchange_with_an_error(tmp_path):
    res = _run("raise", tmp_path)
    assert "injected failure" in res[1].get("error", "")
    assert "error" in res[0], "the surviving rank returned from the exchange without its peer"
    assert res[0]["seconds"] < PG_TIMEOUT_S + 30


def test_a_rank_that_never_joins_times_out_the_exchange(tmp_path):
    res = _run("absent", tmp_path)
    assert res[1].get("absent")
    assert "error" in res[0], "the exchange completed without one rank"
    assert res[0]["seconds"] < PG_TIMEOUT_S + 30


def test_a_late_rank_delays_the_exchange_without_changing_it(tmp_path):
    (tmp_path / "ok").mkdir()
    (tmp_path / "late").mkdir()
    ok = _run("ok", tmp_path / "ok")
    late = _run("delay", tmp_path / "late")
    for r in late:
        assert "error" not in r, r
    assert late[0]["seconds"] >= PG_TIMEOUT_S / 2 - 0.5  # rank 0 waited for its peer
    for key in ("mean", "var", "bsum"):
        assert late[0][key] == ok[0][key] == late[1][key]
