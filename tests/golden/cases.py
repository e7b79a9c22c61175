"""The reference's gputest cases (src/gputest.zig:86-480) plus the ops gputest never checks,
as data: inputs from the seeded generator, one runner for the host-emulated reference
kernels and one for the C oracle, and the comparison class of every output.

Comparison classes (why each is what it is):
  exact  -- both compute the same float operations in the same order: bit patterns equal
            (value equality where the reference kernel writes -0.0 as x*(x>0) and the CPU
            code writes +0.0 by a select: relu)
  tol    -- the reference kernel differs from the CPU code by design, at the ulp level:
            tree vs sequential sums (reductions), x/(sqrt(v)+eps) vs x*(1/(sqrt(v)+eps))
            (normalize), delta*1/sqrt vs delta*(1/sqrt) (normalize_delta), a different
            tanh formula, SELU's constant rounded from two f32 literals, multiply-adds the
            compiler fuses (ramp, the scaled resampling shortcut).
"""
from __future__ import annotations

import ctypes as C

import numpy as np

from darknet_zig_b200 import synth

N_ELEM = 4099  # gputest.zig:87, deliberately not a multiple of the block size
BN = (4, 17, 53)  # gputest.zig:157-159
SOFTMAX = (8, 137)  # gputest.zig:253-254
POOL = (3, 6, 14, 14, 2, 2, 1)  # gputest.zig:393-399: batch, c, h, w, size, stride, pad
POOL_OVERLAP = (2, 3, 13, 13, 3, 2, 2)
SHORTCUT = (2, 8, 8, 4)  # gputest.zig:454-457: batch, w, h, c

ACTS = list(range(14))
TOL_ACTS = {4, 5, 13}  # ramp (x*(x>0) + .1f*x is contracted to one fma), tanh, selu

_f = C.POINTER(C.c_float)
_i = C.POINTER(C.c_int32)


def fp(a):
    return a.ctypes.data_as(_f)


def ip(a):
    return a.ctypes.data_as(_i)


def inputs():
    d = {}
    d["a"] = synth.uniform(101, (N_ELEM,), -1, 1)
    d["b"] = synth.uniform(102, (N_ELEM,), -1, 1)
    B, Cc, S = BN
    d["bn_x"] = synth.uniform(103, (B * Cc * S,), -1, 1)
    d["bn_delta"] = synth.uniform(104, (B * Cc * S,), -1, 1)
    d["bn_bias"] = synth.uniform(105, (Cc,), -1, 1)
    d["bn_scale"] = synth.uniform(106, (Cc,), 0.5, 1.5)
    rb, rc = SOFTMAX
    d["sm_x"] = synth.uniform(107, (rb * rc,), -1, 1)
    d["sm_truth"] = synth.one_hot(108, rb, rc).ravel()
    pb, pc, ph, pw = POOL[:4]
    d["pool_x"] = synth.uniform(109, (pb * pc * ph * pw,), -1, 1)
    ob, oc, oh, ow = POOL_OVERLAP[:4]
    d["pool2_x"] = synth.uniform(110, (ob * oc * oh * ow,), -1, 1)
    sb, sw, sh, sc = SHORTCUT
    d["sc_add"] = synth.uniform(111, (sb * sc * sh * sw,), -1, 1)
    d["sc_out"] = synth.uniform(112, (sb * sc * sh * sw,), -1, 1)
    d["sc2_add"] = synth.uniform(113, (sb * 8 * 16 * 16,), -1, 1)  # 16x16x8 -> 8x8x4 resample
    d["sc2_out"] = synth.uniform(114, (sb * sc * sh * sw,), -1, 1)
    return d


def pool_out(h, w, size, stride, pad):
    return (h + pad - size) // stride + 1, (w + pad - size) // stride + 1


def _act_inputs(d, act):
    """gradient() takes activation outputs (gputest.zig:141-145): y = activate(a)."""
    return d["a"]


def run_reference(emu, d):
    """Outputs of the reference's own kernels (host emulation, gpu.zig argument order)."""
    o = {}
    n = N_ELEM
    x = d["b"].copy(); emu.axpy(n, C.c_float(2.5), fp(d["a"]), fp(x)); o["axpy"] = x
    x = d["a"].copy(); emu.scal(n, C.c_float(0.3), fp(x)); o["scal"] = x
    x = d["b"].copy(); emu.mul(n, fp(d["a"]), fp(x)); o["mul"] = x
    x = d["a"].copy(); emu.add_scalar(n, C.c_float(0.7), fp(x)); o["add_scalar"] = x
    x = d["a"].copy(); emu.constrain(n, C.c_float(0.5), fp(x)); o["constrain"] = x
    x = np.zeros(n, np.float32); emu.fill(n, C.c_float(1.25), fp(x)); o["fill"] = x
    x = np.zeros(n, np.float32); emu.copy(n, fp(d["a"]), fp(x)); o["copy"] = x
    for act in ACTS:
        y = d["a"].copy(); emu.activate_array(fp(y), n, act); o[f"activate_{act}"] = y
        g = d["b"].copy(); emu.gradient_array(fp(y), n, act, fp(g)); o[f"gradient_{act}"] = g
    B, Cc, S = BN
    x = d["bn_x"].copy(); emu.add_bias(fp(x), fp(d["bn_bias"]), B, Cc, S); o["add_bias"] = x
    x = d["bn_x"].copy(); emu.scale_bias(fp(x), fp(d["bn_scale"]), B, Cc, S); o["scale_bias"] = x
    u = np.zeros(Cc, np.float32); emu.backward_bias(fp(u), fp(d["bn_delta"]), B, Cc, S); o["backward_bias"] = u
    m = np.zeros(Cc, np.float32); emu.mean(fp(d["bn_x"]), B, Cc, S, fp(m)); o["mean"] = m
    # downstream ops consume the CPU statistics, so each comparison isolates one kernel
    return o


def run_reference_bn(emu, d, mean, var):
    """BN kernels that take statistics, fed the oracle's statistics."""
    o = {}
    B, Cc, S = BN
    v = np.zeros(Cc, np.float32); emu.variance(fp(d["bn_x"]), fp(mean), B, Cc, S, fp(v)); o["variance"] = v
    xn = d["bn_x"].copy(); emu.normalize(fp(xn), fp(mean), fp(var), B, Cc, S); o["normalize"] = xn
    su = np.zeros(Cc, np.float32)
    emu.backward_scale(fp(xn), fp(d["bn_delta"]), B, Cc, S, fp(su)); o["backward_scale"] = su
    md = np.zeros(Cc, np.float32); emu.mean_delta(fp(d["bn_delta"]), fp(var), B, Cc, S, fp(md)); o["mean_delta"] = md
    vd = np.zeros(Cc, np.float32)
    emu.variance_delta(fp(d["bn_x"]), fp(d["bn_delta"]), fp(mean), fp(var), B, Cc, S, fp(vd)); o["variance_delta"] = vd
    nd = d["bn_delta"].copy()
    emu.normalize_delta(fp(d["bn_x"]), fp(mean), fp(var), fp(md), fp(vd), B, Cc, S, fp(nd)); o["normalize_delta"] = nd
    return o


def run_reference_rest(emu, d):
    o = {}
    rb, rc = SOFTMAX
    sm = np.zeros(rb * rc, np.float32)
    emu.softmax(fp(d["sm_x"]), rc, rb, rc, 1, rc, 1, C.c_float(1.0), fp(sm)); o["softmax"] = sm
    de = np.zeros_like(sm); er = np.zeros_like(sm)
    emu.softmax_x_ent(rb * rc, fp(sm), fp(d["sm_truth"]), fp(de), fp(er)); o["xent_delta"] = de; o["xent_err"] = er
    for key, (pb, pc, ph, pw, size, stride, pad) in (("pool", POOL), ("pool2", POOL_OVERLAP)):
        oh, ow = pool_out(ph, pw, size, stride, pad)
        out_n = pb * pc * oh * ow
        out = np.zeros(out_n, np.float32); idx = np.zeros(out_n, np.int32)
        emu.forward_maxpool(out_n, ph, pw, pc, stride, size, pad, fp(d[f"{key}_x"]), fp(out), ip(idx))
        o[f"{key}_max"] = out; o[f"{key}_idx"] = idx
        delta = synth.uniform(120 if key == "pool" else 121, (out_n,), -1, 1)
        prev = np.zeros(pb * pc * ph * pw, np.float32)
        emu.backward_maxpool(prev.size, ph, pw, pc, stride, size, pad, fp(delta), fp(prev), ip(idx))
        o[f"{key}_back"] = prev
    pb, pc, ph, pw = POOL[:4]
    avg = np.zeros(pb * pc, np.float32)
    emu.forward_avgpool(pb * pc, pw, ph, pc, fp(d["pool_x"]), fp(avg)); o["avgpool"] = avg
    ad = synth.uniform(122, (pb * pc,), -1, 1)
    ind = np.zeros(pb * pc * ph * pw, np.float32)
    emu.backward_avgpool(pb * pc, pw, ph, pc, fp(ind), fp(ad)); o["avgpool_back"] = ind
    sb, sw, sh, sc = SHORTCUT
    out = d["sc_out"].copy()
    emu.shortcut(sb, sw, sh, sc, fp(d["sc_add"]), sw, sh, sc, C.c_float(1.0), C.c_float(1.0), fp(out))
    o["shortcut"] = out
    out = d["sc2_out"].copy()
    emu.shortcut(sb, 16, 16, 8, fp(d["sc2_add"]), sw, sh, sc, C.c_float(0.5), C.c_float(1.5), fp(out))
    o["shortcut_resample"] = out
    return o


def run_oracle(orc, d):
    """The same ops through the C restatement; returns (outputs, bn statistics)."""
    o = {}
    x = d["b"].copy(); orc.axpy(2.5, d["a"], x); o["axpy"] = x
    x = d["a"].copy(); orc.scal(0.3, x); o["scal"] = x
    x = d["b"].copy(); orc.mul(d["a"], x); o["mul"] = x
    x = d["a"].copy(); orc.add_scalar(0.7, x); o["add_scalar"] = x
    x = d["a"].copy(); orc.constrain(0.5, x); o["constrain"] = x
    x = np.zeros(N_ELEM, np.float32); orc.fill(x, 1.25); o["fill"] = x
    x = np.zeros(N_ELEM, np.float32); orc.copy(d["a"], x); o["copy"] = x
    for act in ACTS:
        y = d["a"].copy(); orc.activate_array(y, act); o[f"activate_{act}"] = y
        g = d["b"].copy(); orc.gradient_array(y, act, g); o[f"gradient_{act}"] = g
    B, Cc, S = BN
    x = d["bn_x"].copy(); orc.add_bias(x, d["bn_bias"], B, Cc, S); o["add_bias"] = x
    x = d["bn_x"].copy(); orc.scale_bias(x, d["bn_scale"], B, Cc, S); o["scale_bias"] = x
    u = np.zeros(Cc, np.float32); orc.backward_bias(u, d["bn_delta"], B, Cc, S); o["backward_bias"] = u
    m = np.zeros(Cc, np.float32); orc.mean(d["bn_x"], B, Cc, S, m); o["mean"] = m
    v = np.zeros(Cc, np.float32); orc.variance(d["bn_x"], m, B, Cc, S, v); o["variance"] = v
    xn = d["bn_x"].copy(); orc.normalize(xn, m, v, B, Cc, S); o["normalize"] = xn
    su = np.zeros(Cc, np.float32); orc.backward_scale(xn, d["bn_delta"], B, Cc, S, su); o["backward_scale"] = su
    md = np.zeros(Cc, np.float32); orc.mean_delta(d["bn_delta"], v, B, Cc, S, md); o["mean_delta"] = md
    vd = np.zeros(Cc, np.float32); orc.variance_delta(d["bn_x"], d["bn_delta"], m, v, B, Cc, S, vd)
    o["variance_delta"] = vd
    nd = d["bn_delta"].copy(); orc.normalize_delta(d["bn_x"], m, v, md, vd, B, Cc, S, nd); o["normalize_delta"] = nd
    rb, rc = SOFTMAX
    sm = np.zeros(rb * rc, np.float32); orc.softmax(d["sm_x"], rc, rb, rc, 1, rc, 1, 1.0, sm); o["softmax"] = sm
    de = np.zeros_like(sm); er = np.zeros_like(sm)
    orc.softmax_cross_entropy(sm, d["sm_truth"], de, er); o["xent_delta"] = de; o["xent_err"] = er
    for key, (pb, pc, ph, pw, size, stride, pad) in (("pool", POOL), ("pool2", POOL_OVERLAP)):
        oh, ow = pool_out(ph, pw, size, stride, pad)
        out_n = pb * pc * oh * ow
        out = np.zeros(out_n, np.float32); idx = np.zeros(out_n, np.int32)
        orc.forward_maxpool(pb, ph, pw, pc, stride, size, pad, d[f"{key}_x"], out, idx)
        o[f"{key}_max"] = out; o[f"{key}_idx"] = idx
        delta = synth.uniform(120 if key == "pool" else 121, (out_n,), -1, 1)
        prev = np.zeros(pb * pc * ph * pw, np.float32)
        orc.backward_maxpool(delta, idx, prev)
        o[f"{key}_back"] = prev
    pb, pc, ph, pw = POOL[:4]
    avg = np.zeros(pb * pc, np.float32); orc.forward_avgpool(pb, pc, ph, pw, d["pool_x"], avg); o["avgpool"] = avg
    ad = synth.uniform(122, (pb * pc,), -1, 1)
    ind = np.zeros(pb * pc * ph * pw, np.float32); orc.backward_avgpool(pb, pc, ph, pw, ad, ind)
    o["avgpool_back"] = ind
    sb, sw, sh, sc = SHORTCUT
    out = d["sc_out"].copy(); orc.shortcut(sb, sw, sh, sc, d["sc_add"], sw, sh, sc, 1.0, 1.0, out)
    o["shortcut"] = out
    out = d["sc2_out"].copy(); orc.shortcut(sb, 16, 16, 8, d["sc2_add"], sw, sh, sc, 0.5, 1.5, out)
    o["shortcut_resample"] = out
    return o, (m, v)


def comparison_class(key: str) -> str:
    if key in ("backward_bias", "mean", "variance", "normalize", "backward_scale", "mean_delta", "variance_delta",
               "normalize_delta", "shortcut_resample"):
        return "tol"
    if key.startswith("activate_") and int(key.split("_")[1]) in TOL_ACTS:
        return "tol"
    if key.startswith("gradient_") and int(key.split("_")[1]) in TOL_ACTS:
        return "tol"
    if key == "activate_1":  # relu: -0.0 vs +0.0
        return "value"
    return "exact"


def run_reference_all(emu, orc, d):
    o = run_reference(emu, d)
    _, (m, v) = run_oracle(orc, d)
    o.update(run_reference_bn(emu, d, m, v))
    o.update(run_reference_rest(emu, d))
    return o
