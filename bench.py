"""Benchmark: one data-parallel training step of a batchnorm + leaky layer
by default (config 0+1 with --config 01).

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--config 4|01] [--shape B,C,H,W] [--sgd-weights N]

A step (config 4, per GPU):
    forward  sync-BN + leaky(0.1) train forward   (read x, write y: 8 B/elem compulsory)
    backward sync-BN + leaky backward             (read delta and x, write dx: 12 B/elem)
    update   SGD momentum 0.9, decay 5e-4         (read w and wu, write both: 16 B/weight)
on NCHW fp32 [128,256,28,28] per GPU (25.7 M elements, 98 MiB per tensor) and a 64 Mi-float
weight vector. With N GPUs every rank holds its own 128-image shard and the per-channel
statistics span all ranks (sync-BN, global batch 128*N; the fused kernels exchange them over
NVLink themselves): weak scaling. N = 1 runs the same step on one GPU (the single-GPU fused
kernels). `--config 01` is BASELINE configs 0+1: [128,128,32,32], forward + backward, no
update.

Before timing, every rank runs one step and checks it (`parity` in the line): the global
per-channel mean and variance against a float64 recomputation over all ranks' shards
(1e-5 relative / 1e-6 absolute, relative to max(|exact|, the terms' 2-norm / n)); mean,
variance and rolling statistics bit-identical on every rank; y and dx bit-identical to a
float32 recomputation from the kernels' own per-channel values (numpy, one IEEE rounding per
operation, as the reference's strict-mode CPU code); the backward sums within the same bar
of float64; SGD bit-exact on a sample of weights (exact rational arithmetic for the fused
multiply-adds). A failed check prints the line with `parity` = "failed: ..." and exits 1.

Timing: W untimed steps, then timed regions of K launches each: K whole steps (forward on
set k, backward on set k+1, then the update), K forwards, K backwards, K updates. Every
kernel starts with a cold L2: the launches rotate through sets of (x, delta, y, dx) that
together exceed twice the 126 MB L2 and the weight vectors are 512 MiB, so each kernel also
writes back its predecessor's dirty outputs, as in a training step. The launches of a region
run back to back between one pair of CUDA events on the launching stream (a GPU-side spin
before the region lets the host queue them all first); a barrier and a synchronize bracket
each region and the times are the maximum over ranks. `--flush read|write` instead runs an
untimed read (or write) of a 256 MiB buffer before each launch and brackets every launch with
its own events; `--flush none` gives the warm-L2 figure (one tensor set, back to back).
`value` is the algorithmic bytes of all ranks per step divided by the step time.

`e2e` repeats the step through the C ABI with HOST buffers: x and delta are copied in from
pinned memory and y and dx copied out every step, inside the timed region (the weights stay
resident on the device, as in training).

`--impl reference` times the reference's CPU implementation of the same step (the C
restatement of blas.zig / batchnorm.zig / activations.zig / convolutional.zig's update in
oracle/, the reference's own Zig code having no toolchain here) on all host cores. Where a
GPU and the reference's own kernel file built for sm_100a (oracle/_ref/libref_gpu.so) are
present, its line also carries `gpu_kernels`: the reference's unfused GPU layer sequences (12
launches forward, 7 backward, 3 for the update, with the reference's grids) timed on the same
workload the same way as this library's step.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time
from fractions import Fraction

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

LEAKY = 7
BYTES_FWD = 8   # per element: read x, write y
BYTES_BWD = 12  # per element: read delta, read x, write dx
BYTES_SGD = 16  # per weight: read w, wu; write w, wu
HBM_NOMINAL_GBS = 8000.0  # BASELINE metric's "% of 8 TB/s"
SGD_LR, SGD_MOMENTUM, SGD_DECAY = 0.1, 0.9, 5e-4

CONFIGS = {
    "4": {"shape": (128, 256, 28, 28), "sgd_weights": 64 << 20},
    "01": {"shape": (128, 128, 32, 32), "sgd_weights": 0},
}


def parse(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=30)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--config", choices=sorted(CONFIGS), default="4",
                    help="BASELINE config: 4 = sync-BN step + SGD (default), 01 = BN forward + backward")
    ap.add_argument("--shape", default="", help="per-GPU batch,channels,height,width (overrides the config's)")
    ap.add_argument("--sgd-weights", type=int, default=-1, help="weights of the SGD update (0: no update)")
    ap.add_argument("--flush", choices=["rotate", "read", "write", "none"], default="rotate",
                    help="cold L2 for every timed kernel: rotate through sets of tensors larger than L2 "
                         "together, with no flush kernel (each kernel also writes back the previous "
                         "one's dirty outputs, as in a training step); or read a 256 MiB buffer before "
                         "each kernel (L2 left clean); or write one (L2 left full of dirty lines). "
                         "'none' is the warm-L2 figure: the same tensors every launch, back to back")
    ap.add_argument("--syncbn", choices=["fused", "split"], default="fused",
                    help="N > 1: statistics exchanged inside the fused kernels over NVLink (fused) or by "
                         "NCCL collectives between split kernels (split)")
    ap.add_argument("--ops", action="store_true",
                    help="instead of the step: time every other op of the path at its BASELINE config shape, "
                         "one JSON line per op")
    ap.add_argument("--op", default="", help="with --ops: only the ops whose name contains this")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-parity", action="store_true", help="skip the pre-timing parity check")
    ap.add_argument("--full-dp", action="store_true",
                    help="instead of the step: the data-parallel weight update of config 4 (gradient "
                         "reduce-scatter, fused SGD on each rank's shard, all-gather of the weights)")
    ap.add_argument("--dp-impl", choices=["fused", "nccl"], default="fused",
                    help="--full-dp: one kernel per rank over NVLink peer memory (fused) or NCCL "
                         "reduce-scatter / all-gather around the library's SGD kernels (nccl)")
    a = ap.parse_args(argv)
    a.warmup = max(a.warmup, 3)
    cfg = CONFIGS[a.config]
    a.shape = tuple(int(v) for v in a.shape.split(",")) if a.shape else cfg["shape"]
    a.sgd_weights = cfg["sgd_weights"] if a.sgd_weights < 0 else a.sgd_weights
    return a


def workload_desc(a, n):
    B, C, H, W = a.shape
    if a.config == "4":
        head = "BASELINE cfg4: data-parallel sync-BN training step"
    else:
        head = "BASELINE cfg0+cfg1: BN-train forward + leaky(0.1) then BN+leaky backward"
    s = (f"{head}, NCHW fp32 [{B},{C},{H},{W}] per GPU, global batch {B * n}"
         + (f", per-channel statistics synchronised over {n} GPUs" if n > 1 else ", 1 GPU")
         + "; sync-BN+leaky(0.1) forward, backward")
    if a.sgd_weights:
        s += (f", then SGD (momentum {SGD_MOMENTUM}, decay {SGD_DECAY}, lr {SGD_LR}) on "
              f"{a.sgd_weights / 2**20:.0f} Mi fp32 weights per GPU")
    return s


def step_bytes(a, E):
    """Algorithmic bytes of one rank's step."""
    return (BYTES_FWD + BYTES_BWD) * E + BYTES_SGD * a.sgd_weights


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profiled_traffic():
    """ncu DRAM bytes per launch of the kernels, from the committed summary."""
    p = os.path.join(ROOT, "profiles", "bn_traffic.json")
    if os.path.exists(p):
        try:
            return json.load(open(p))
        except Exception:
            return None
    return None


# ---- clocks ---------------------------------------------------------------------------

class ClockSampler:
    """SM clock and clock-event reasons during the timed regions: `nvidia-smi -lms` in its own
    process (read-only queries; a process of its own, so no Python thread scheduling thins
    the samples), with one NVML reading as the fallback."""

    FIELDS = ("clocks.sm", "clocks.max.sm", "clocks_event_reasons.hw_slowdown",
              "clocks_event_reasons.hw_thermal_slowdown", "clocks_event_reasons.sw_thermal_slowdown",
              "clocks_event_reasons.sw_power_cap")
    REASONS = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")

    def __init__(self, gpu_index: int, interval_ms: int = 10):
        self.idx = gpu_index
        self.interval_ms = interval_ms
        self.proc = None
        self.out = None

    def _target(self) -> str:
        try:
            import torch

            return "GPU-" + str(torch.cuda.get_device_properties(self.idx).uuid)
        except Exception:
            return str(self.idx)

    def start(self):
        import tempfile

        self.out = tempfile.TemporaryFile(mode="w+")
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", self._target(), "--query-gpu=" + ",".join(self.FIELDS),
                 "--format=csv,noheader,nounits", "-lms", str(self.interval_ms)],
                stdout=self.out, stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None
            return
        # the timed regions start once the tool prints (its start-up takes longer on boxes with
        # more GPUs); give up after 5 s and fall back to one reading after the regions
        deadline = time.time() + 5.0
        while time.time() < deadline and self.proc.poll() is None:
            self.out.flush()
            if os.fstat(self.out.fileno()).st_size > 0:
                break
            time.sleep(0.02)

    def stop(self):
        rows = []
        if self.proc is not None:
            time.sleep(2 * self.interval_ms / 1000)
            self.proc.terminate()  # the sampler started above, by its own handle
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
                self.proc.wait()
            self.out.seek(0)
            for line in self.out:
                parts = [v.strip() for v in line.split(",")]
                if len(parts) != len(self.FIELDS):
                    continue
                try:
                    rows.append((float(parts[0]), float(parts[1]), parts[2:]))
                except ValueError:
                    continue
        if self.out is not None:
            self.out.close()
        if not rows:
            return self._nvml_once()
        reasons = sorted({name for _, _, flags in rows for name, f in zip(self.REASONS, flags) if f == "Active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_min_mhz": min(r[0] for r in rows),
                "sm_max_mhz": max(r[1] for r in rows), "reasons": reasons, "samples": len(rows),
                "interval_ms": self.interval_ms, "source": "nvidia-smi -lms during the timed regions"}

    def _nvml_once(self):
        try:
            import pynvml

            pynvml.nvmlInit()
            h = pynvml.nvmlDeviceGetHandleByIndex(self.idx)
            sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
            smax = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            return {"sm_mhz": float(sm), "sm_max_mhz": float(smax), "reasons": [], "samples": 1,
                    "source": "nvml, once after the timed regions"}
        except Exception:
            return None


# ---- parity of one step (plain numpy / torch float64 checker; not the library) -------------

def round_f32(v: Fraction) -> np.float32:
    """The float32 nearest to the rational v, ties to even."""
    f = np.float32(float(v))
    best = None
    for c in (np.nextafter(f, np.float32(-np.inf)), f, np.nextafter(f, np.float32(np.inf))):
        if not np.isfinite(c):
            continue
        err = abs(Fraction(float(c)) - v)
        key = (err, int(np.array(c).view(np.uint32)) & 1)
        if best is None or key < best[0]:
            best = (key, c)
    return best[1]


def fma_f32(a, b, c) -> np.float32:
    """fmaf(a, b, c) with a single rounding."""
    return round_f32(Fraction(float(a)) * Fraction(float(b)) + Fraction(float(c)))


def leaky_f32(t):
    return np.where(t > np.float32(0), t, np.float32(0.1) * t)


def check_step_parity(dist, world, B, C, S, x, delta, y, dx, gamma, beta, mean, var, rm0, rv0, rm, rv, bu, su, md, vd,
                      w0, wu0, w, wu, sgd_batch):
    """Checks one step's results on this rank (see the module docstring). Returns
    (ok, detail); every rank takes the same collective steps in the same order."""
    import torch

    f32 = np.float32
    fails = []
    n_total = B * S * world
    # global statistics in float64 over every rank's shard
    xd = x.view(B, C, S).double()
    s1 = xd.sum(dim=(0, 2))
    sq = (xd * xd).sum(dim=(0, 2))
    if dist:
        dist.all_reduce(s1)
        dist.all_reduce(sq)
    mu = s1 / n_total
    dev2 = (xd - mu[None, :, None]) ** 2
    m2 = dev2.sum(dim=(0, 2))
    q = (dev2 * dev2).sum(dim=(0, 2))
    del dev2, xd
    if dist:
        dist.all_reduce(m2)
        dist.all_reduce(q)
    var_exact = m2 / (n_total - 1)

    def close(got, want, scale, name):
        got = got.double()
        bound = 1e-6 + 1e-5 * torch.maximum(want.abs(), scale)
        err = (got - want).abs()
        plain = float((err / want.abs().clamp_min(1e-30)).max())
        if bool((err > bound).any()):
            fails.append(f"{name}: max err/bound {float((err / bound).max()):.3g}")
        return plain

    rel = {"mean": close(mean, mu, sq.sqrt() / n_total, "mean"),
           "variance": close(var, var_exact, q.sqrt() / (n_total - 1), "variance")}
    # the statistics and rolling statistics are identical on every rank
    if dist:
        mine = torch.cat([mean, var, rm, rv]).view(torch.int32)
        allv = [torch.empty_like(mine) for _ in range(world)]
        dist.all_gather(allv, mine)
        if any(not torch.equal(v, allv[0]) for v in allv):
            fails.append("per-channel statistics differ between ranks")
    m = mean.cpu().numpy()
    v = var.cpu().numpy()
    rm_w = np.array([fma_f32(f32(1) - f32(0.99), m[c], rm0[c] * f32(0.99)) for c in range(C)], f32)
    rv_w = np.array([fma_f32(f32(1) - f32(0.99), v[c], rv0[c] * f32(0.99)) for c in range(C)], f32)
    if not (np.array_equal(rm.cpu().numpy().view(np.uint32), rm_w.view(np.uint32))
            and np.array_equal(rv.cpu().numpy().view(np.uint32), rv_w.view(np.uint32))):
        fails.append("rolling statistics not bit-exact")
    # per-element outputs from the kernels' per-channel values, in slabs of images
    g = gamma.cpu().numpy()[None, :, None]
    b = beta.cpu().numpy()[None, :, None]
    inv = (f32(1) / (np.sqrt(v) + f32(0.000001)))[None, :, None]
    inv2 = (f32(1) / np.sqrt(v + f32(0.00001)))[None, :, None]
    mdv = md.cpu().numpy()
    vdv = vd.cpu().numpy()[None, :, None]
    denom = f32(n_total)
    mdd = (mdv / denom)[None, :, None]
    mc = m[None, :, None]
    g1 = np.zeros(C, np.float64)
    g2 = np.zeros(C, np.float64)
    g1s = np.zeros(C, np.float64)
    g2s = np.zeros(C, np.float64)
    y_bad = dx_bad = 0
    step = max(1, (1 << 22) // (C * S))
    for n0 in range(0, B, step):
        n1 = min(B, n0 + step)
        xs = x.view(B, C, S)[n0:n1].cpu().numpy()
        ds = delta.view(B, C, S)[n0:n1].cpu().numpy()
        yw = leaky_f32((xs - mc) * inv * g + b)
        y_bad += int((y.view(B, C, S)[n0:n1].cpu().numpy().view(np.uint32) != yw.view(np.uint32)).sum())
        gr = ds * np.where(yw > f32(0), f32(1), f32(0.1))
        dxw = (gr * g) * inv2 + (vdv * f32(2) * (xs - mc)) / denom + mdd
        dx_bad += int((dx.view(B, C, S)[n0:n1].cpu().numpy().view(np.uint32) != dxw.view(np.uint32)).sum())
        gd = gr.astype(np.float64)
        t2 = gd * (xs.astype(np.float64) - mc.astype(np.float64))
        g1 += gd.sum(axis=(0, 2))
        g2 += t2.sum(axis=(0, 2))
        g1s += (gd * gd).sum(axis=(0, 2))
        g2s += (t2 * t2).sum(axis=(0, 2))
    if y_bad:
        fails.append(f"y: {y_bad} elements not bit-exact")
    if dx_bad:
        fails.append(f"dx: {dx_bad} elements not bit-exact")
    sums = torch.from_numpy(np.stack([g1, g2, g1s, g2s])).to(x.device)
    if dist:
        dist.all_reduce(sums)
    s_g, s_gx, s_gs, s_gxs = (t for t in sums)
    rel["bias_updates"] = close(bu, s_g, s_gs.sqrt(), "bias_updates (sum g)")
    inv_t = torch.from_numpy(inv.ravel().astype(np.float64)).to(x.device)
    rel["scale_updates"] = close(su, s_gx * inv_t, s_gxs.sqrt() * inv_t, "scale_updates (sum g x_norm)")
    # SGD: exact fused multiply-adds on a sample of weights
    if w0 is not None:
        b32 = f32(sgd_batch)
        a_decay = f32(-f32(SGD_DECAY) * b32)
        a_lr = f32(f32(SGD_LR) / b32)
        rng = np.random.default_rng(7)
        idx = np.sort(rng.choice(w.numel(), size=2048, replace=False))
        it = torch.from_numpy(idx).to(w.device)
        w_got = w[it].cpu().numpy()
        u_got = wu[it].cpu().numpy()
        bad = 0
        for k in range(idx.size):
            u1 = fma_f32(a_decay, w0[k], wu0[k])
            w1 = fma_f32(a_lr, u1, w0[k])
            u2 = f32(u1 * f32(SGD_MOMENTUM))
            bad += int(np.float32(w1).view(np.uint32) != w_got[k].view(np.uint32)
                       or np.float32(u2).view(np.uint32) != u_got[k].view(np.uint32))
        if bad:
            fails.append(f"sgd: {bad} of {idx.size} sampled weights not bit-exact")
    ok = torch.tensor([0 if fails else 1], device=x.device)
    if dist:
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
    detail = {"max_rel_err_vs_exact": {k: float(f"{v:.3g}") for k, v in rel.items()},
              "checked": "global mean/variance vs float64 over all ranks; statistics identical on every rank; "
                         "rolling statistics, y, dx bit-exact; backward sums vs float64"
                         + ("; SGD bit-exact on 2048 sampled weights" if w0 is not None else "")}
    if fails:
        detail["rank_failures"] = fails
    return bool(ok.item()), detail


# ---- our implementation -----------------------------------------------------------------

def run_ours(a):
    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != a.gpus:
        raise SystemExit(f"--gpus {a.gpus} but WORLD_SIZE={world}")
    torch.cuda.set_device(local)
    from darknet_zig_b200 import gpu, syncbn

    gpu.init(local)
    dist = None
    if world > 1:
        import datetime

        import torch.distributed as td

        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist = td
    B, C, H, W = a.shape
    S = H * W
    E = B * C * S
    NW = a.sgd_weights
    sgd_batch = B * world
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    # rotate: enough sets of (x, delta, y, dx) that a step's tensors were last touched more
    # than two L2 capacities (2 x 126 MB) of traffic earlier
    n_sets = 1 if a.flush != "rotate" else max(2, -(-(3 * 126 * 2**20) // (4 * E * 4)) + 1)
    back_to_back = a.flush in ("rotate", "none")
    sets = []
    for _ in range(n_sets):
        sx = torch.randn(E, generator=g, device=dev)
        sd = torch.randn(E, generator=g, device=dev)
        sets.append((sx, sd, torch.empty_like(sx), torch.empty_like(sx)))
    x, delta, y, dx = sets[0]
    # the layer's parameters and running statistics are replicated, as in data-parallel
    # training: the same values on every rank (only the batch shards differ)
    gw = torch.Generator(device=dev)
    gw.manual_seed(99)
    gamma = torch.rand(C, generator=gw, device=dev) + 0.5
    beta = torch.randn(C, generator=gw, device=dev) * 0.1
    mean, var, bu, su, md, vd = (torch.zeros(C, device=dev) for _ in range(6))
    rm = torch.randn(C, generator=gw, device=dev) * 0.5
    rv = torch.rand(C, generator=gw, device=dev) * 1.5 + 0.5
    wts = torch.randn(NW, generator=gw, device=dev) * 0.01 if NW else None
    wup = torch.randn(NW, generator=gw, device=dev) * 1e-3 if NW else None
    flush_buf = torch.ones(64 << 20, dtype=torch.float32, device=dev) if not back_to_back else None

    def flush():
        if a.flush == "read":
            flush_buf.sum()
        elif a.flush == "write":
            flush_buf.fill_(1.0)

    layer = syncbn.SyncBN(B, C, S, world=world, dist=dist, fused=a.syncbn == "fused", rank=rank)

    def fwd(k):
        sx, sd, sy, sdx = sets[k % n_sets]
        layer.forward(sx, sy, gamma, beta, mean, var, rm, rv, LEAKY)

    def bwd(k):
        # the backward of a step works on the next set: its x was last touched a whole
        # rotation earlier, as a layer's backward comes long after its forward
        sx, sd, sy, sdx = sets[(k + 1) % n_sets]
        layer.backward(sx, sd, sdx, gamma, beta, mean, var, bu, su, md, vd, LEAKY)

    def sgd(k):
        if NW:
            gpu.sgdMomentum(NW, wts, wup, SGD_LR, SGD_MOMENTUM, SGD_DECAY, sgd_batch)

    def whole(k):
        fwd(k)
        bwd(k)
        sgd(k)

    # one checked step on set 0 (forward and backward on the same tensors, as a layer does)
    parity = "skipped (--no-parity)"
    parity_detail = None
    if not a.no_parity:
        rm0, rv0 = rm.cpu().numpy(), rv.cpu().numpy()
        w0 = wu0 = None
        if NW:
            rs = np.random.default_rng(7)
            idx = np.sort(rs.choice(NW, size=2048, replace=False))
            it = torch.from_numpy(idx).to(dev)
            w0, wu0 = wts[it].cpu().numpy(), wup[it].cpu().numpy()
        bu.zero_()
        su.zero_()
        layer.forward(x, y, gamma, beta, mean, var, rm, rv, LEAKY)
        layer.backward(x, delta, dx, gamma, beta, mean, var, bu, su, md, vd, LEAKY)
        sgd(0)
        torch.cuda.synchronize()
        gpu.check_device_error()
        ok, parity_detail = check_step_parity(dist, world, B, C, S, x, delta, y, dx, gamma, beta, mean, var, rm0, rv0,
                                              rm, rv, bu, su, md, vd, w0, wu0, wts, wup, sgd_batch)
        parity = "ok" if ok else "failed: " + "; ".join(parity_detail.get("rank_failures", ["on another rank"]))

    stream = torch.cuda.current_stream()
    for k in range(a.warmup):
        flush()
        fwd(k)
        flush()
        bwd(k)
        flush()
        sgd(k)
    torch.cuda.synchronize()
    gpu.check_device_error()

    def timed(body):
        """Device time of body(k) for k < steps, in ms per k (max over ranks by the caller).
        A GPU-side spin first lets the host queue every launch before the GPU reaches them,
        so no interval contains time the GPU waited for the host."""
        if dist:
            dist.barrier()
        torch.cuda.synchronize()
        torch.cuda._sleep(int(0.25e-3 * 2e9) * a.steps)
        if back_to_back:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for k in range(a.steps):
                body(k)
            e1.record(stream)
            torch.cuda.synchronize()
            return e0.elapsed_time(e1) / a.steps
        ev = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
        for k in range(a.steps):
            flush()
            ev[k][0].record(stream)
            body(k)
            ev[k][1].record(stream)
        torch.cuda.synchronize()
        return sum(e0.elapsed_time(e1) for e0, e1 in ev) / a.steps

    clocks = ClockSampler(local)
    clocks.start()
    launches0 = gpu.launch_count()
    if back_to_back:
        ms_step = timed(whole)
    launches = gpu.launch_count() - launches0
    ms_fwd = timed(fwd)
    ms_bwd = timed(bwd)
    ms_sgd = timed(sgd) if NW else 0.0
    if not back_to_back:
        ms_step = ms_fwd + ms_bwd + ms_sgd
        launches = gpu.launch_count() - launches0
    if dist:
        dist.barrier()
    clk = clocks.stop()
    gpu.check_device_error()
    if dist:
        t = torch.tensor([ms_step, ms_fwd, ms_bwd, ms_sgd], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms_step, ms_fwd, ms_bwd, ms_sgd = (float(v) for v in t.cpu())

    e2e = None
    if not a.no_e2e:
        e2e = run_e2e(a, layer, x, y, delta, dx, gamma, beta, mean, var, rm, rv, bu, su, md, vd, sgd, dev, dist, world)

    torch.cuda.synchronize()
    layer.close()
    if dist:
        # release NCCL state before the process group goes away
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        if parity.startswith("failed"):
            raise SystemExit(1)
        return
    peak, peak_kind = measured_peaks()
    bytes_step = step_bytes(a, E) * world
    value = bytes_step / (ms_step * 1e-3) / 1e9
    # the committed ncu traffic belongs to the default workload only
    traffic = (profiled_traffic() or {}) if (a.config == "4" and a.shape == CONFIGS["4"]["shape"]) else {}
    kernels = {
        "bn_act_forward_train": (ms_fwd, BYTES_FWD * E, "sync-BN+leaky forward" if world > 1 else "BN+leaky forward"),
        "bn_act_backward": (ms_bwd, BYTES_BWD * E, "sync-BN+leaky backward" if world > 1 else "BN+leaky backward"),
    }
    if NW:
        kernels["sgd_momentum"] = (ms_sgd, BYTES_SGD * NW, "fused SGD update")
    kout = {}
    for name, (ms, nbytes, what) in kernels.items():
        gbs = nbytes / (ms * 1e-3) / 1e9
        kout[name] = {"what": what, "ms": round(ms, 5), "GBps": round(gbs, 1), "frac_of_peak": round(gbs / peak, 4),
                      "algorithmic_bytes": nbytes, "launches": 1}
    dom = max(kernels, key=lambda k: kernels[k][0])
    dms, dbytes, _ = kernels[dom]
    dgbs = dbytes / (dms * 1e-3) / 1e9
    line = {
        "metric": "training-step HBM throughput of the BN+leaky layer (algorithmic bytes / device time)",
        "value": round(value, 2),
        "unit": "GB/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms_step, 5),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (torch.randn / rand; batch shards seeded per rank, parameters and weights identical on every rank)",
        "parity": parity,
        "config": {"workload": workload_desc(a, world), "baseline_config": a.config, "batch_per_gpu": B,
                   "channels": C, "hw": [H, W], "global_batch": B * world, "activation": "leaky 0.1",
                   "sgd_weights_per_gpu": NW,
                   "l2": (f"rotating {n_sets} sets of (x, delta, y, dx), {n_sets * 4 * E * 4 / 2**20:.0f} MiB, "
                          f"and {2 * NW * 4 / 2**20:.0f} MiB of weights: every kernel starts cold and writes back "
                          f"its predecessor's outputs" if a.flush == "rotate" else
                          "warm L2: the same (x, delta, y, dx) every launch, back to back (not the "
                          "headline)" if a.flush == "none" else
                          f"256 MiB buffer {'read' if a.flush == 'read' else 'written'} before every timed "
                          f"kernel (cold L2{'' if a.flush == 'read' else ', full of dirty lines'})")
                         + f"; {E * 4 / 2**20:.0f} MiB tensors",
                   "parallelism": f"dp{world}" + (f" + sync-BN ({a.syncbn})" if world > 1 else "")},
        "bytes_per_step_per_gpu": step_bytes(a, E),
        "elems_per_s": round(E * world / (ms_step * 1e-3), 1),
        "pct_of_8TBs": round(100.0 * value / world / HBM_NOMINAL_GBS, 2),
        "kernels": kout,
        "roofline": {"kernel": dom, "bound": "hbm", "achieved": round(dgbs, 1), "peak": peak,
                     "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)" if peak_kind == "measured"
                     else "fallback 6.65 TB/s", "unit": "GB/s", "frac": round(dgbs / peak, 4),
                     "traffic": (traffic.get(dom) or {}).get("dram_bytes_per_launch"),
                     "algorithmic_bytes": dbytes},
        "gpu_launches": launches,
        "clocks": clk,
    }
    if parity_detail:
        line["parity_detail"] = parity_detail
    if e2e:
        line["e2e"] = e2e
    if not a.no_cpu_baseline and world == 1:
        line["cpu_baseline"] = cpu_baseline(a, threads=1)
    print(json.dumps(line), flush=True)
    if parity.startswith("failed"):
        raise SystemExit(1)


def run_e2e(a, layer, x, y, delta, dx, gamma, beta, mean, var, rm, rv, bu, su, md, vd, sgd, dev, dist, world):
    """The step through the C ABI with host buffers: every step copies its x and delta in
    from pinned host memory, runs the forward, backward and update, and copies y and dx back
    out, all inside the timed region. Copies in, kernels and copies out run on three streams
    over two device buffer sets, so step k's outputs travel to the host while step k+1's
    inputs travel in (PCIe is full duplex) and step k+1 computes; the time is from the
    first copy in to the last copy out."""
    import torch

    E = x.numel()
    hx = torch.empty(E, dtype=torch.float32, pin_memory=True)
    hd = torch.empty(E, dtype=torch.float32, pin_memory=True)
    hy = torch.empty(E, dtype=torch.float32, pin_memory=True)
    hdx = torch.empty(E, dtype=torch.float32, pin_memory=True)
    hx.copy_(x.cpu())
    hd.copy_(delta.cpu())
    bufs = [(x, delta, y, dx), tuple(torch.empty_like(x) for _ in range(4))]
    s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
    ev_in = [torch.cuda.Event() for _ in bufs]
    ev_run = [torch.cuda.Event() for _ in bufs]
    ev_out = [torch.cuda.Event() for _ in bufs]
    steps = max(3, min(a.steps, 30))  # the window's first copy in and last copy out do not overlap

    def step(k):
        b = k % len(bufs)
        bx, bd, by, bdx = bufs[b]
        s_in.wait_event(ev_run[b])  # the kernels of step k-2 have read this set's inputs
        with torch.cuda.stream(s_in):
            bx.copy_(hx, non_blocking=True)
            bd.copy_(hd, non_blocking=True)
        ev_in[b].record(s_in)
        s_run.wait_event(ev_in[b])
        s_run.wait_event(ev_out[b])  # step k-2's outputs have left this set
        with torch.cuda.stream(s_run):
            layer.forward(bx, by, gamma, beta, mean, var, rm, rv, LEAKY)
            layer.backward(bx, bd, bdx, gamma, beta, mean, var, bu, su, md, vd, LEAKY)
            sgd(k)
        ev_run[b].record(s_run)
        s_out.wait_event(ev_run[b])
        with torch.cuda.stream(s_out):
            hy.copy_(by, non_blocking=True)
            hdx.copy_(bdx, non_blocking=True)
        ev_out[b].record(s_out)

    for k in range(2 * len(bufs)):
        step(k)
    torch.cuda.synchronize()
    if dist:
        dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record(s_in)
    for k in range(steps):
        step(k)
    e.record(s_out)
    torch.cuda.synchronize()
    ms = s.elapsed_time(e) / steps
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    value = step_bytes(a, E) * world / (ms * 1e-3) / 1e9
    return {"value": round(value, 2), "unit": "GB/s", "ms_per_step": round(ms, 4), "steps": steps,
            "h2d_bytes_per_step": 2 * E * 4, "d2h_bytes_per_step": 2 * E * 4,
            "path": "C ABI with pinned host buffers; copies in, kernels and copies out on three streams over "
                    "two device buffer sets (steps pipelined); weights resident on the device",
            "pcie": pcie_bound(hx, hd, hy, hdx, bufs[1], s_in, s_out, steps)}


def pcie_bound(hx, hd, hy, hdx, dbuf, s_in, s_out, reps):
    """What the host link alone allows for one step's copies (no kernels): the two inputs in,
    the two outputs out, and both directions at once, each timed with events over `reps`
    repetitions. The last is the floor of the end-to-end step time."""
    import torch

    bx, bd, by, bdx = dbuf
    n = 2 * hx.numel() * 4

    def timed(ins, outs):
        torch.cuda.synchronize()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        s_in.wait_event(s)
        s_out.wait_event(s)
        for _ in range(reps):
            if ins:
                with torch.cuda.stream(s_in):
                    bx.copy_(hx, non_blocking=True)
                    bd.copy_(hd, non_blocking=True)
            if outs:
                with torch.cuda.stream(s_out):
                    hy.copy_(by, non_blocking=True)
                    hdx.copy_(bdx, non_blocking=True)
        torch.cuda.current_stream().wait_stream(s_in)
        torch.cuda.current_stream().wait_stream(s_out)
        e.record()
        torch.cuda.synchronize()
        return s.elapsed_time(e) / reps

    t_in, t_out, t_both = timed(True, False), timed(False, True), timed(True, True)
    return {"h2d_GBps": round(n / (t_in * 1e-3) / 1e9, 2), "d2h_GBps": round(n / (t_out * 1e-3) / 1e9, 2),
            "both_directions_ms": round(t_both, 4),
            "note": "copies of one step alone; both_directions_ms is the floor of the e2e step time"}


# ---- the reference's CPU implementation -----------------------------------------------------

def cpu_step_sample(a, threads, steps, warmup, images=None):
    """Times the reference's op sequence (oracle restatement) for one training step of the
    workload: BN+leaky forward and backward over `images` images of the per-GPU shape (all
    of them by default), then the SGD update of the config's weights. Returns (seconds per
    step, elements, weights)."""
    from darknet_zig_b200 import synth
    from oracle.oracle import Oracle

    orc = Oracle()
    orc.set_threads(threads)
    B, C, H, W = a.shape
    B = images or B
    S = H * W
    E = B * C * S
    NW = a.sgd_weights
    x = synth.normal(1, (E,), 0, 1)
    d0 = synth.normal(2, (E,), 0, 1)
    gamma = synth.uniform(3, (C,), 0.5, 1.5)
    beta = synth.normal(4, (C,), 0, 0.1)
    y = np.zeros(E, np.float32)
    xs = np.zeros(E, np.float32)
    xn = np.zeros(E, np.float32)
    z = lambda: np.zeros(C, np.float32)  # noqa: E731
    mean, var, rm, rv, bu, su, md, vd = (z() for _ in range(8))
    w = synth.normal(5, (NW,), 0, 0.01) if NW else None
    wu = synth.normal(6, (NW,), 0, 1e-3) if NW else None
    times = []
    for i in range(warmup + steps):
        delta = d0.copy()
        t0 = time.perf_counter()
        orc.bn_forward_layer(x, y, xs, xn, B, C, S, gamma, beta, mean, var, rm, rv, True, LEAKY)
        orc.bn_backward_layer(xs, xn, y, delta, B, C, S, gamma, mean, var, bu, su, md, vd, LEAKY)
        if NW:
            orc.sgd_update(w, wu, SGD_LR, SGD_MOMENTUM, SGD_DECAY, B)
        t1 = time.perf_counter()
        if i >= warmup:
            times.append(t1 - t0)
    return sum(times) / len(times), E, NW


def cpu_model() -> str:
    """The host CPU's model name (/proc/cpuinfo), for the baseline lines."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown CPU"


def cpu_baseline(a, threads):
    # a bounded sample: as many full steps as fit ~10 s at this core count (at least 2)
    t_one, E, NW = cpu_step_sample(a, threads, 1, 0)
    steps = int(max(2, min(20, 10.0 / max(t_one, 1e-3))))
    t, E, NW = cpu_step_sample(a, threads, steps, 1)
    gbs = ((BYTES_FWD + BYTES_BWD) * E + BYTES_SGD * NW) / t / 1e9
    return {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{steps} full steps of the workload (BN+leaky fwd+bwd over {E} elements"
                      + (f", SGD on {NW} weights" if NW else "") + f") through the C restatement of the "
                      f"reference CPU ops; {t * 1e3:.1f} ms/step; host {os.cpu_count()} cpus ({cpu_model()})",
            "ms_per_step": round(t * 1e3, 2), "elems_per_s": round(E / t, 1)}


def ref_gpu_kernels(a):
    """The reference's GPU path on this box's GPU 0: darknet_kernels.hip compiled for sm_100a
    with the reference's flags, launched with the reference's grids (oracle/ref_gpu.cu). One
    step = the conv-layer BN + leaky forward sequence (convolutional.zig:263-268,
    batchnorm.zig:129-153), backward sequence (convolutional.zig:279-282,
    batchnorm.zig:155-170) and the weight update (convolutional.zig:332-334). Timed like this
    library's step: rotating tensor sets larger than L2 together, K back-to-back steps
    between one pair of events after W warm-up steps. Returns None when there is no GPU or
    the library was not built."""
    try:
        import torch
    except ImportError:
        return None
    if not torch.cuda.is_available():
        return None
    try:
        from oracle.oracle import RefGpu

        ref = RefGpu()
    except (FileNotFoundError, OSError) as e:
        return {"unavailable": f"reference kernel library: {e}"}
    torch.cuda.set_device(0)
    B, C, H, W = a.shape
    S = H * W
    E = B * C * S
    NW = a.sgd_weights
    g = torch.Generator(device="cuda")
    g.manual_seed(4321)
    # per set: the conv output (forward in place), the saved x and x_norm, delta (backward in place)
    n_sets = max(2, -(-(3 * 126 * 2**20) // (4 * E * 4)) + 1)
    sets = [tuple(torch.randn(E, generator=g, device="cuda") for _ in range(4)) for _ in range(n_sets)]
    gamma = torch.rand(C, generator=g, device="cuda") + 0.5
    beta = torch.randn(C, generator=g, device="cuda") * 0.1
    mean, var, rm, rv, bu, su, md, vd = (torch.zeros(C, device="cuda") for _ in range(8))
    w = torch.randn(NW, generator=g, device="cuda") * 0.01 if NW else None
    wu = torch.randn(NW, generator=g, device="cuda") * 1e-3 if NW else None
    stream = torch.cuda.current_stream()
    sh = stream.cuda_stream
    P = lambda t: t.data_ptr()  # noqa: E731

    def fwd(k):
        out, xs, xn, _ = sets[k % n_sets]
        ref.conv_bn_forward(P(out), P(xs), P(xn), P(mean), P(var), P(rm), P(rv), P(gamma), P(beta), B, C, S,
                            LEAKY, sh)

    def bwd(k):
        out, xs, xn, delta = sets[(k + 1) % n_sets]
        ref.conv_bn_backward(P(out), P(delta), P(xs), P(xn), P(mean), P(var), P(gamma), P(bu), P(su), P(md), P(vd),
                             B, C, S, LEAKY, sh)

    def sgd(k):
        if NW:
            ref.sgd_weights(NW, SGD_LR, SGD_MOMENTUM, SGD_DECAY, B, P(w), P(wu), sh)

    def timed(body, steps):
        torch.cuda.synchronize()
        torch.cuda._sleep(int(2e-3 * 2e9) * max(1, steps // 4))
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(steps):
            body(k)
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / steps

    for k in range(a.warmup):
        fwd(k)
        bwd(k)
        sgd(k)
    torch.cuda.synchronize()
    ms_step = timed(lambda k: (fwd(k), bwd(k), sgd(k)), a.steps)
    ms_fwd = timed(fwd, a.steps)
    ms_bwd = timed(bwd, a.steps)
    ms_sgd = timed(sgd, a.steps) if NW else 0.0
    del sets, w, wu
    torch.cuda.empty_cache()
    gbs = lambda nbytes, ms: round(nbytes / (ms * 1e-3) / 1e9, 1)  # noqa: E731
    return {
        "what": "the reference's darknet_kernels.hip built for sm_100a (nvcc -O3, its build.zig flags), "
                "launched with its own grids (gpu.zig:420-477) on GPU 0 of this box, 1 GPU",
        "ms_per_step": round(ms_step, 5),
        "value": gbs(step_bytes(a, E), ms_step),
        "unit": "GB/s (this workload's algorithmic bytes / device time)",
        "forward_ms": round(ms_fwd, 5),
        "backward_ms": round(ms_bwd, 5),
        "sgd_ms": round(ms_sgd, 5),
        "launches_per_step": ref.launches_forward + ref.launches_backward + (ref.launches_sgd if NW else 0),
        "l2": f"rotating {n_sets} sets of 4 tensors ({n_sets * 4 * E * 4 / 2**20:.0f} MiB)",
    }


def run_reference(a):
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    threads = len(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else (os.cpu_count() or 1)
    B, C, H, W = a.shape
    gpu_kernels = ref_gpu_kernels(a)
    t, E, NW = cpu_step_sample(a, threads, a.steps, min(a.warmup, 3))
    gbs = ((BYTES_FWD + BYTES_BWD) * E + BYTES_SGD * NW) / t / 1e9
    line = {
        "impl": "reference",
        "metric": "training-step HBM throughput of the BN+leaky layer (algorithmic bytes / device time)",
        "value": round(gbs, 3),
        "unit": "GB/s",
        "n_gpus": a.gpus,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(t * 1e3, 3),
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (seeded splitmix64 generator)",
        # the same workload string as this library's line at the same --gpus; the host computes one
        # rank's shard (the reference has no multi-GPU path), whose GB/s is the step's rate
        "config": {"workload": workload_desc(a, a.gpus), "baseline_config": a.config, "batch_per_gpu": B,
                   "channels": C, "hw": [H, W], "sgd_weights_per_gpu": NW,
                   "parallelism": "host cores (reference CPU ops, OpenMP over channels / elements), one "
                                  "rank's shard"},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{a.steps} full steps (after {min(a.warmup, 3)} warm-up) of the reference op "
                                   f"sequence batchnorm.zig:74-123 + activations.zig"
                                   + (" + convolutional.zig:217-233's update" if NW else "")
                                   + f", C restatement in oracle/; {threads} threads of {cpu_model()}"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "elems_per_s": round(E / t, 1),
    }
    if gpu_kernels is not None:
        line["gpu_kernels"] = gpu_kernels
    print(json.dumps(line), flush=True)


# ---- the other ops of the path -----------------------------------------------------------

def run_ops(a):
    """Device time of every other op at its BASELINE config shape (1 GPU): back-to-back
    launches over rotating buffer sets larger than L2 together, CUDA events around them;
    GB/s = algorithmic bytes (each tensor read or written once) / time."""
    import torch

    from darknet_zig_b200 import gpu

    torch.cuda.set_device(0)
    gpu.init(0)
    peak, _ = measured_peaks()
    stream = torch.cuda.current_stream()
    steps = max(a.steps, 10)

    def timed(name, config, nbytes, make, run):
        if a.op and a.op not in name:
            return
        n_sets = int(min(8, max(2, -(-(3 * 126 * 2**20) // max(nbytes, 1)) + 1)))
        sets = [make(i) for i in range(n_sets)]
        for k in range(a.warmup):
            run(sets[k % n_sets])
        torch.cuda.synchronize()
        torch.cuda._sleep(int(0.1e-3 * 2e9) * steps)
        l0 = gpu.launch_count()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for k in range(steps):
            run(sets[k % n_sets])
        e1.record(stream)
        torch.cuda.synchronize()
        launches = (gpu.launch_count() - l0) / steps
        gpu.check_device_error()
        us = e0.elapsed_time(e1) / steps * 1e3
        gbs = nbytes / (us * 1e-6) / 1e9
        print(json.dumps({"op": name, "config": config, "us": round(us, 2), "GBps": round(gbs, 1),
                          "frac_of_peak": round(gbs / peak, 4), "algorithmic_bytes": int(nbytes),
                          "launches_per_call": launches, "rotating_sets": n_sets}), flush=True)

    f32 = dict(dtype=torch.float32, device="cuda")
    LEAKY_ = LEAKY
    # cfg2: inference BN + leaky over the tiny-classifier stack, N=64; maxpool 2x2/s2 between stages
    stack = [(16, 224), (32, 112), (64, 56), (128, 28), (256, 14), (512, 7), (1024, 7)]
    for c, hw in stack:
        E = 64 * c * hw * hw

        def make_bn(i, E=E, c=c):
            return (torch.randn(E, **f32), torch.empty(E, **f32), torch.rand(c, **f32) + 0.5, torch.randn(c, **f32),
                    torch.randn(c, **f32), torch.rand(c, **f32) + 0.5)

        timed("bn_act_forward_infer", f"cfg2 64x{c}x{hw}x{hw} leaky", 8 * E, make_bn,
              lambda t, c=c, hw=hw: gpu.bnActForwardInfer(t[0], t[1], 64, c, hw * hw, t[2], t[3], t[4], t[5], LEAKY_))
    for c, hw in stack[:5]:
        E = 64 * c * hw * hw
        On = E // 4

        def make_mp(i, E=E, On=On):
            return (torch.randn(E, **f32), torch.empty(On, **f32), torch.empty(On, dtype=torch.int32, device="cuda"))

        timed("forward_maxpool", f"cfg2 64x{c}x{hw}x{hw} 2x2/s2 with indices", 4 * E + 8 * On, make_mp,
              lambda t, c=c, hw=hw, On=On: gpu.forwardMaxpool(On, hw, hw, c, 2, 2, 1, t[0], t[1], t[2]))
    # cfg3: classifier head at N=256
    E = 256 * 1000 * 49
    timed("forward_avgpool", "cfg3 256x1000x7x7", 4 * E + 4 * 256 * 1000,
          lambda i: (torch.randn(E, **f32) * 2, torch.empty(256 * 1000, **f32)),
          lambda t: gpu.forwardAvgpool(256 * 1000, 7, 7, 1000, t[0], t[1]))

    def make_sx(i):
        truth = torch.zeros(256, 1000, **f32)
        truth[torch.arange(256), torch.randint(0, 1000, (256,))] = 1.0
        return (torch.randn(256 * 1000, **f32), truth.view(-1), torch.empty(256 * 1000, **f32),
                torch.empty(256 * 1000, **f32), torch.empty(256 * 1000, **f32), torch.zeros(1, **f32))

    timed("softmax_xent", "cfg3 256 rows x 1000 classes", 16 * 256 * 1000, make_sx,
          lambda t: gpu.softmaxXent(t[0], t[1], 1000, 256, 1.0, t[2], t[3], t[4], t[5]))
    E = 256 * 512 * 196
    timed("shortcut", "cfg3 256x512x14x14 + same shape", 12 * E,
          lambda i: (torch.randn(E, **f32), torch.randn(E, **f32)),
          lambda t: gpu.shortcut(256, 14, 14, 512, t[0], 14, 14, 512, 1.0, 1.0, t[1]))
    # cfg4: SGD momentum on the 64 Mi weight vector; BN + leaky per GPU at 128x256x28x28
    n = 64 << 20
    timed("sgd_momentum", "cfg4 64 Mi weights, lr 0.1 momentum 0.9 decay 5e-4 batch 1024", 16 * n,
          lambda i: (torch.randn(n, **f32) * 0.01, torch.randn(n, **f32) * 1e-3),
          lambda t: gpu.sgdMomentum(n, t[0], t[1], 0.1, 0.9, 5e-4, 1024))
    for (b_, c_, s_, label) in ((128, 256, 784, "cfg4 per GPU 128x256x28x28"), (128, 128, 1024, "cfg0/1 128x128x32x32"),
                                (64, 1024, 49, "64x1024x7x7"), (16, 40, 169, "16x40x13x13")):
        E = b_ * c_ * s_

        def make_bnt(i, E=E, c_=c_):
            return (torch.randn(E, **f32), torch.empty(E, **f32), torch.randn(E, **f32), torch.empty(E, **f32),
                    torch.rand(c_, **f32) + 0.5, torch.randn(c_, **f32) * 0.1,
                    *(torch.zeros(c_, **f32) for _ in range(8)))

        timed("bn_act_forward_train", f"{label} leaky", 8 * E, make_bnt,
              lambda t, b_=b_, c_=c_, s_=s_: gpu.bnActForwardTrain(t[0], t[1], None, b_, c_, s_, t[4], t[5], t[6],
                                                                   t[7], t[8], t[9], LEAKY_))
        timed("bn_act_backward", f"{label} leaky", 12 * E, make_bnt,
              lambda t, b_=b_, c_=c_, s_=s_: gpu.bnActBackward(t[0], None, t[2], t[3], b_, c_, s_, t[4], t[5], t[6],
                                                               t[7], t[10], t[11], t[12], t[13], LEAKY_))
        if s_ % 4 == 0:
            # the forward from a producer's statistics: one (count, mean, M2) per 128-pixel tile
            # and channel, as a GEMM epilogue would leave them; x read once, y written once
            npc = -(-(b_ * s_) // 128)

            def make_fs(i, E=E, c_=c_, npc=npc, n_=b_ * s_):
                pc = torch.zeros((npc, c_, 3), dtype=torch.float64, device="cuda")
                pc[:, :, 0] = 128.0
                pc[-1, :, 0] = float(n_ - 128 * (npc - 1))
                pc[:, :, 2] = pc[:, :, 0]
                return (torch.randn(E, **f32), torch.empty(E, **f32), pc, torch.rand(c_, **f32) + 0.5,
                        torch.randn(c_, **f32) * 0.1, *(torch.zeros(c_, **f32) for _ in range(4)))

            timed("bn_act_forward_from_stats", f"{label} leaky, {npc} tiles of statistics", 8 * E + 24 * npc * c_,
                  make_fs, lambda t, b_=b_, c_=c_, s_=s_, npc=npc: gpu.bnActForwardFromStats(
                      t[0], t[1], None, b_, c_, s_, t[2], npc, t[3], t[4], t[5], t[6], t[7], t[8], LEAKY_))
    # the BLAS-1 basics on 64 Mi floats
    timed("fill", "64 Mi floats", 4 * n, lambda i: (torch.empty(n, **f32),), lambda t: gpu.fill(t[0], n, 0.5))
    timed("copy", "64 Mi floats", 8 * n, lambda i: (torch.randn(n, **f32), torch.empty(n, **f32)),
          lambda t: gpu.copy(n, t[0], t[1]))
    timed("axpy", "64 Mi floats", 12 * n, lambda i: (torch.randn(n, **f32), torch.randn(n, **f32)),
          lambda t: gpu.axpy(n, 0.5, t[0], t[1]))


def run_full_dp(a):
    """Config 4's weight update in full data parallelism (darknet_zig_b200/dpsgd.py) on the
    64 Mi-float weight vector: each step sums the ranks' gradients of this rank's shard, adds
    them into its momentum shard, applies the fused SGD, and gives every rank the updated
    weights. --dp-impl fused: one kernel per rank over NVLink peer memory (dnb_dpsgd_step);
    nccl: NCCL reduce-scatter, this library's axpy + SGD kernels, NCCL all-gather. Before
    timing one step is checked: weights bit-identical on every rank, and a sample of 2048
    weights equal to the update with the gradients summed in float32 in rank order (exact for
    the fused kernel and for two ranks; within 1e-6 relative for NCCL with more ranks, whose
    sum order NCCL chooses)."""
    import datetime

    import torch

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    from darknet_zig_b200 import gpu
    from darknet_zig_b200.dpsgd import FusedShardedSGD, ShardedSGD

    gpu.init(local)
    dist = None
    if world > 1:
        import torch.distributed as td

        td.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
        dist = td
    dev = torch.device("cuda", local)
    n = a.sgd_weights or (64 << 20)
    batch = a.shape[0] * world
    fused = a.dp_impl == "fused"
    gw = torch.Generator(device=dev)
    gw.manual_seed(99)
    gr = torch.Generator(device=dev)
    gr.manual_seed(500 + rank)
    if fused:
        opt = FusedShardedSGD(n, world, rank, dist=dist)
        w = opt.weights
        w[:n].copy_(torch.randn(n, generator=gw, device=dev) * 0.01)
        opt.grads[:n].copy_(torch.randn(n, generator=gr, device=dev) * 1e-3)
        grads = [opt.grads, opt.grads]  # read by the step, never written: one buffer serves every step
        torch.cuda.synchronize()
        if dist:
            dist.barrier()

        def do_step(g):
            opt.step(SGD_LR, SGD_MOMENTUM, SGD_DECAY, batch)
    else:
        opt = ShardedSGD(n, world, rank, dist=dist, device=dev)
        w = opt.padded(torch.randn(n, generator=gw, device=dev) * 0.01)
        grads = [opt.padded(torch.randn(n, generator=gr, device=dev) * 1e-3) for _ in range(2)]

        def do_step(g):
            opt.step(w, g, SGD_LR, SGD_MOMENTUM, SGD_DECAY, batch)
    # one checked step
    idx = torch.from_numpy(np.sort(np.random.default_rng(3).choice(n, size=2048, replace=False))).to(dev)
    w0 = w[idx].cpu().numpy()
    g_all = [torch.empty(2048, device=dev) for _ in range(world)]
    if dist:
        dist.all_gather(g_all, grads[0][idx].contiguous())
    else:
        g_all = [grads[0][idx]]
    g_sum = np.zeros(2048, np.float32)
    for gq in g_all:
        g_sum = (g_sum + gq.cpu().numpy()).astype(np.float32)
    do_step(grads[0])
    torch.cuda.synchronize()
    gpu.check_device_error()
    fails = []
    w1 = w[idx].cpu().numpy()
    b32 = np.float32(batch)
    a_decay = np.float32(-np.float32(SGD_DECAY) * b32)
    a_lr = np.float32(np.float32(SGD_LR) / b32)
    bad = 0
    for k in range(2048):
        u1 = fma_f32(a_decay, w0[k], g_sum[k])  # the momentum shard starts at 0: wu = sum of gradients
        want = fma_f32(a_lr, u1, w0[k])
        if world <= 2 or fused:
            bad += int(np.float32(want).view(np.uint32) != w1[k].view(np.uint32))
        else:
            bad += int(abs(float(want) - float(w1[k])) > 1e-6 * max(abs(float(want)), 1e-30))
    if bad:
        fails.append(f"{bad} of 2048 sampled weights off the expected update")
    if dist:
        # a checksum of every weight's bits
        hs = w[:n].view(torch.int32).to(torch.int64).sum().reshape(1)
        allh = [torch.empty_like(hs) for _ in range(world)]
        dist.all_gather(allh, hs)
        if any(not torch.equal(h, allh[0]) for h in allh):
            fails.append("weights differ between ranks")
        ok = torch.tensor([0 if fails else 1], device=dev)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN)
        passed = bool(ok.item())
    else:
        passed = not fails
    for k in range(a.warmup):
        do_step(grads[k % 2])
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    clocks = ClockSampler(local)
    clocks.start()
    if dist:
        dist.barrier()
    torch.cuda.synchronize()
    torch.cuda._sleep(int(1e-3 * 2e9) * max(1, a.steps // 4))
    l0 = gpu.launch_count()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for k in range(a.steps):
        do_step(grads[k % 2])
    e1.record(stream)
    torch.cuda.synchronize()
    launches = gpu.launch_count() - l0
    ms = e0.elapsed_time(e1) / a.steps
    clk = clocks.stop()
    gpu.check_device_error()
    if fused:
        opt.close()
    if dist:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    shard = opt.shard
    line = {
        "metric": "full data-parallel weight update of the layer's 64 Mi weights (gradient reduce-scatter, "
                  "fused SGD on each rank's shard, weight all-gather): weights updated per second",
        "impl_variant": ("one kernel per rank over NVLink peer memory (dnb_dpsgd_step)" if fused else
                         "NCCL reduce-scatter + dnb_axpy + dnb_sgd_momentum + NCCL all-gather"),
        "value": round(n / (ms * 1e-3), 1),
        "unit": "weights/s",
        "n_gpus": world,
        "steps": a.steps,
        "warmup": a.warmup,
        "ms_per_step": round(ms, 5),
        "higher_is_better": True,
        "scaling": "strong",
        "vs_baseline": None,
        "dtype": "f32",
        "data": "synthetic (torch.randn; gradients seeded per rank, weights identical on every rank)",
        "parity": "ok" if passed else "failed: " + "; ".join(fails or ["on another rank"]),
        "config": {"workload": f"BASELINE cfg4 weight update, full data parallelism over {world} GPU(s): "
                               f"{n} fp32 gradients summed over the ranks shard by shard, momentum SGD "
                               f"(momentum {SGD_MOMENTUM}, decay {SGD_DECAY}, lr {SGD_LR}, global batch {batch}) "
                               f"on {shard} weights per rank, the weights gathered on every rank "
                               f"({'fused kernel over NVLink' if fused else 'NCCL collectives'})",
                   "momentum": "sharded (each rank keeps its 1/N)", "parallelism": f"dp{world}"},
        "hbm_bytes_per_rank_step": 28 * shard,
        "collective_bytes_per_rank_step": 2 * 4 * shard * (world - 1),
        "gpu_launches": launches,
        "clocks": clk,
    }
    print(json.dumps(line), flush=True)
    if not passed:
        raise SystemExit(1)


def main():
    a = parse()
    if a.full_dp:
        run_full_dp(a)
        return
    if a.ops:
        run_ops(a)
        return
    if a.impl == "reference":
        run_reference(a)
    else:
        run_ours(a)


if __name__ == "__main__":
    main()
