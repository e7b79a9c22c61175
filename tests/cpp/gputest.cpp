// CPU-vs-GPU comparison through the C++ host mirror (darknet_zig_b200/host/gpu.hpp), in the
// shape of the reference's `darknet-zig gputest` (gputest.zig:58-84): each op runs on the
// CPU twin and on the device over the same seeded input, and one line per check reports the
// largest absolute and relative difference. The CPU twins are the oracle's C restatement of
// the reference CPU ops (oracle/ref_ops.c, test infrastructure). The bars are this build's,
// tighter than gputest's 1e-3 (gputest.zig:29): bit-identical for the exact class
// (elementwise, bias/scale, relu/leaky/linear, maxpool values and indices, shortcut, SGD),
// 1e-5 relative / 1e-6 absolute for reductions and transcendentals.
//
//     gputest          run every check on device 0 (exit 1 if any fails)
//     gputest --list   print the checks without touching a device
//
// Shapes follow gputest.zig: n = 4099 (gputest.zig:87), batch 4 x filters 17 x spatial 53
// (:157-159), 8 rows x 137 classes (:253-254), pool 3 x 6 x 14 x 14, 2x2 / 2 / pad 1
// (:393-399), shortcut 2 x 8 x 8 x 4 (:454-457); the fused entries add the bench shape's
// smaller sibling.
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <cstring>
#include <functional>
#include <string>
#include <vector>

#include "gpu.hpp"
#include "ref_ops.h"

namespace {

namespace g = dnb::gpu;
using Vec = std::vector<float>;

int failures = 0, checks = 0;
bool list_only = false;

enum Bar { Exact, Tol };

// One check: max abs / rel difference, and the bar. For Tol, the relative error of a
// reduction is taken against max(|cpu|, scale) (scale: the 2-norm of the summed terms, or 0).
void report(const char *name, const Vec &cpu, const Vec &dev, Bar bar, const Vec *scale = nullptr) {
    ++checks;
    double max_abs = 0.0, max_rel = 0.0;
    bool ok = cpu.size() == dev.size();
    for (size_t i = 0; ok && i < cpu.size(); ++i) {
        const double a = cpu[i], b = dev[i];
        const double d = std::fabs(a - b);
        double ref = std::fabs(a);
        if (scale) ref = std::max(ref, (double)(*scale)[i]);
        max_abs = std::max(max_abs, d);
        if (ref > 0) max_rel = std::max(max_rel, d / ref);
        if (bar == Exact) {
            uint32_t ua, ub;
            std::memcpy(&ua, &cpu[i], 4);
            std::memcpy(&ub, &dev[i], 4);
            if (ua != ub) ok = false;
        } else if (d > 1e-6 + 1e-5 * ref) {
            ok = false;
        }
    }
    if (!ok) ++failures;
    std::printf("%-32s %s  %s  max abs diff %12.4e  max rel %12.4e\n", name, ok ? "ok  " : "FAIL",
                bar == Exact ? "bit-exact" : "1e-5 rel ", max_abs, max_rel);
}

// splitmix64 -> uniform floats in [lo, hi)
struct Rng {
    uint64_t s;
    explicit Rng(uint64_t seed) : s(seed) {}
    uint64_t next() {
        uint64_t z = (s += 0x9e3779b97f4a7c15ull);
        z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
        z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
        return z ^ (z >> 31);
    }
    float uniform(float lo, float hi) { return lo + (hi - lo) * (float)((next() >> 40) * (1.0 / 16777216.0)); }
};
Vec random(Rng &r, size_t n, float lo = -1, float hi = 1) {
    Vec v(n);
    for (auto &x : v) x = r.uniform(lo, hi);
    return v;
}
Vec pull(g::Buf b, size_t n) {
    Vec v(n);
    g::pull(b, v.data(), n);
    return v;
}

// device scope guard for a Buf
struct Dev {
    g::Buf b;
    explicit Dev(const Vec &v) : b(g::make(v.data(), v.size())) {}
    explicit Dev(size_t n) : b(g::alloc(n)) {}
    ~Dev() { g::free(b); }
    operator g::Buf() const { return b; }
};

// 2-norm per channel of [batch, filters, spatial] terms
Vec channel_norm(const Vec &t, int64_t B, int64_t C, int64_t S) {
    Vec out(C, 0.0f);
    for (int64_t c = 0; c < C; ++c) {
        double s = 0;
        for (int64_t b = 0; b < B; ++b)
            for (int64_t k = 0; k < S; ++k) s += (double)t[(b * C + c) * S + k] * t[(b * C + c) * S + k];
        out[c] = (float)std::sqrt(s);
    }
    return out;
}

struct Check {
    const char *section;
    std::function<void()> run;
};

void elementwise() {
    const size_t n = 4099;  // deliberately not a multiple of the block size
    Rng rng(20240921);
    const Vec a = random(rng, n), b = random(rng, n);
    {
        Vec cpu = b;
        ref_axpy(2.5f, a.data(), cpu.data(), n);
        Dev da(a), db(b);
        g::axpy(n, 2.5f, da, db);
        report("axpy", cpu, pull(db, n), Exact);
    }
    {
        Vec cpu = a;
        ref_scal(0.3f, cpu.data(), n);
        Dev da(a);
        g::scal(n, 0.3f, da);
        report("scal", cpu, pull(da, n), Exact);
    }
    {
        Vec cpu(n);
        ref_fill(cpu.data(), n, 0.7f);
        Dev da(n);
        g::fill(da, n, 0.7f);
        report("fill", cpu, pull(da, n), Exact);
    }
    {
        Vec cpu(n);
        ref_copy(a.data(), cpu.data(), n);
        Dev da(a), db(n);
        g::copy(n, da, db);
        report("copy", cpu, pull(db, n), Exact);
    }
    {
        Vec cpu = b;
        ref_mul(a.data(), cpu.data(), n);
        Dev da(a), db(b);
        g::mul(n, da, db);
        report("mul", cpu, pull(db, n), Exact);
    }
    {
        Vec cpu = a;
        ref_constrain(0.5f, cpu.data(), n);
        Dev da(a);
        g::constrain(n, 0.5f, da);
        report("constrain", cpu, pull(da, n), Exact);
    }
    const struct {
        int act;
        const char *name;
        Bar bar;
    } acts[] = {{g::leaky, "leaky", Exact}, {g::relu, "relu", Exact}, {g::linear, "linear", Exact},
                {g::logistic, "logistic", Tol}};
    for (const auto &ac : acts) {
        Vec cpu = a;
        ref_activate_array(cpu.data(), n, ac.act);
        Dev da(a);
        g::activateArray(da, n, ac.act);
        report((std::string("activate ") + ac.name).c_str(), cpu, pull(da, n), ac.bar);
        Vec grad = b;
        ref_gradient_array(cpu.data(), n, ac.act, grad.data());
        Dev dy(cpu), dd(b);
        g::gradientArray(dy, n, ac.act, dd);
        report((std::string("gradient ") + ac.name).c_str(), grad, pull(dd, n), ac.bar);
    }
}

void biasAndNorm() {
    const int64_t B = 4, C = 17, S = 53, n = B * C * S;
    Rng rng(20240922);
    const Vec x = random(rng, n), delta = random(rng, n), bias = random(rng, C), scale = random(rng, C, 0.5f, 1.5f);
    {
        Vec cpu = x;
        ref_add_bias(cpu.data(), bias.data(), B, C, S);
        Dev dx(x), dbias(bias);
        g::addBias(dx, dbias, B, C, S);
        report("add_bias", cpu, pull(dx, n), Exact);
    }
    {
        Vec cpu = x;
        ref_scale_bias(cpu.data(), scale.data(), B, C, S);
        Dev dx(x), ds(scale);
        g::scaleBias(dx, ds, B, C, S);
        report("scale_bias", cpu, pull(dx, n), Exact);
    }
    const Vec dnorm = channel_norm(delta, B, C, S);
    {
        Vec cpu(C, 0.0f);
        ref_backward_bias(cpu.data(), delta.data(), B, C, S);
        Dev dd(delta), du(C);
        g::backwardBias(du, dd, B, C, S);
        report("backward_bias", cpu, pull(du, C), Tol, &dnorm);
    }
    {
        Vec prod(n);
        for (int64_t i = 0; i < n; ++i) prod[i] = x[i] * delta[i];
        const Vec pn = channel_norm(prod, B, C, S);
        Vec cpu(C, 0.0f);
        ref_backward_scale(x.data(), delta.data(), B, C, S, cpu.data());
        Dev dx(x), dd(delta), du(C);
        g::backwardScale(dx, dd, B, C, S, du);
        report("backward_scale", cpu, pull(du, C), Tol, &pn);
    }
    Vec m(C), v(C);
    ref_mean(x.data(), B, C, S, m.data());
    ref_variance(x.data(), m.data(), B, C, S, v.data());
    {
        Vec sc = channel_norm(x, B, C, S);
        for (auto &t : sc) t /= (float)(B * S);
        Dev dx(x), dm(C);
        g::mean(dx, B, C, S, dm);
        report("mean", m, pull(dm, C), Tol, &sc);
    }
    {
        // the twin's own fp32 rounding is allowed: scale = 2-norm of the squared deviations
        // / (n-1), plus the twin's distance from the float64 variance (as a 1e-5 multiple)
        Vec sc(C);
        for (int64_t c = 0; c < C; ++c) {
            double s1 = 0, s2 = 0, s4 = 0;
            for (int64_t b = 0; b < B; ++b)
                for (int64_t k = 0; k < S; ++k) s1 += x[(b * C + c) * S + k];
            const double mu = s1 / (B * S);
            for (int64_t b = 0; b < B; ++b)
                for (int64_t k = 0; k < S; ++k) {
                    const double d = x[(b * C + c) * S + k] - mu;
                    s2 += d * d;
                    s4 += d * d * d * d;
                }
            const double vex = s2 / (B * S - 1);
            sc[c] = (float)(std::sqrt(s4) / (B * S - 1) + std::fabs(v[c] - vex) / 1e-5);
        }
        Dev dx(x), dm(m), dv(C);
        g::variance(dx, dm, B, C, S, dv);
        report("variance", v, pull(dv, C), Tol, &sc);
    }
    {
        Vec cpu = x;
        ref_normalize(cpu.data(), m.data(), v.data(), B, C, S);
        Dev dx(x), dm(m), dv(v);
        g::normalize(dx, dm, dv, B, C, S);
        report("normalize", cpu, pull(dx, n), Exact);
    }
    Vec md(C), vd(C);
    ref_mean_delta(delta.data(), v.data(), B, C, S, md.data());
    ref_variance_delta(x.data(), delta.data(), m.data(), v.data(), B, C, S, vd.data());
    {
        Vec sc(C);
        for (int64_t c = 0; c < C; ++c) sc[c] = dnorm[c] / std::sqrt(v[c] + 1e-5f);
        Dev dd(delta), dv(v), out(C);
        g::meanDelta(dd, dv, B, C, S, out);
        report("mean_delta", md, pull(out, C), Tol, &sc);
    }
    {
        Dev dx(x), dd(delta), dm(m), dv(v), out(C);
        g::varianceDelta(dx, dd, dm, dv, B, C, S, out);
        // scale: the 2-norm of the summed terms delta*(x-m), times the closing factor
        Vec terms(n);
        for (int64_t b = 0; b < B; ++b)
            for (int64_t c = 0; c < C; ++c)
                for (int64_t k = 0; k < S; ++k) {
                    const int64_t i = (b * C + c) * S + k;
                    terms[i] = delta[i] * (x[i] - m[c]);
                }
        Vec sc = channel_norm(terms, B, C, S);
        for (int64_t c = 0; c < C; ++c) sc[c] *= 0.5f * std::pow(v[c] + 1e-5f, -1.5f);
        report("variance_delta", vd, pull(out, C), Tol, &sc);
    }
    {
        Vec cpu = delta;
        ref_normalize_delta(x.data(), m.data(), v.data(), md.data(), vd.data(), B, C, S, cpu.data());
        Dev dx(x), dm(m), dv(v), dmd(md), dvd(vd), dd(delta);
        g::normalizeDelta(dx, dm, dv, dmd, dvd, B, C, S, dd);
        report("normalize_delta", cpu, pull(dd, n), Exact);
    }
}

void softmaxAndLoss() {
    const int64_t batch = 8, classes = 137, n = batch * classes;
    Rng rng(20240923);
    const Vec x = random(rng, n, -2, 2);
    Vec truth(n, 0.0f);
    for (int64_t b = 0; b < batch; ++b) truth[b * classes + (int64_t)(rng.next() % classes)] = 1.0f;
    Vec p(n);
    ref_softmax(x.data(), classes, batch, classes, 1, classes, 1, 1.0f, p.data());
    {
        Dev dx(x), dp(n);
        g::softmax(dx, classes, batch, classes, 1, classes, 1, 1.0f, dp);
        report("softmax", p, pull(dp, n), Tol);
    }
    Vec d(n), e(n);
    ref_softmax_cross_entropy(p.data(), truth.data(), d.data(), e.data(), n);
    {
        Dev dp(p), dt(truth), dd(n), de(n);
        g::softmaxCrossEntropy(n, dp, dt, dd, de);
        report("softmax_cross_entropy delta", d, pull(dd, n), Exact);
        report("softmax_cross_entropy err", e, pull(de, n), Tol);
    }
    {
        Dev dx(x), dt(truth), dout(n), dd(n), de(n), dc(1);
        g::softmaxXent(dx, dt, classes, batch, 1.0f, dout, dd, de, dc);
        report("softmax_xent output", p, pull(dout, n), Tol);
        report("softmax_xent delta", d, pull(dd, n), Tol);
        report("softmax_xent err", e, pull(de, n), Tol);
        const Vec cost{ref_sum_array(e.data(), n)};
        report("softmax_xent cost", cost, pull(dc, 1), Tol);
    }
}

void pooling() {
    const int64_t B = 3, C = 6, H = 14, W = 14, size = 2, stride = 2, pad = size - 1;
    const int64_t oh = ref_maxpool_out_dim(H, size, stride, pad), ow = ref_maxpool_out_dim(W, size, stride, pad);
    const int64_t in_n = B * C * H * W, out_n = B * C * oh * ow;
    Rng rng(20240924);
    const Vec x = random(rng, in_n);
    Vec out(out_n);
    std::vector<int32_t> idx(out_n);
    ref_forward_maxpool(B, H, W, C, stride, size, pad, x.data(), out.data(), idx.data());
    Dev dx(x), dout(out_n), didx(out_n);
    g::forwardMaxpool(out_n, H, W, C, stride, size, pad, dx, dout, didx);
    report("forward_maxpool values", out, pull(dout, out_n), Exact);
    std::vector<int32_t> gidx(out_n);
    dnb_pull(gidx.data(), didx.b.ptr, sizeof(int32_t) * out_n, nullptr);
    dnb_sync();
    Vec ia(out_n), ib(out_n);
    for (int64_t i = 0; i < out_n; ++i) {
        ia[i] = (float)idx[i];
        ib[i] = (float)gidx[i];
    }
    report("forward_maxpool indexes", ia, ib, Exact);
    const Vec delta = random(rng, out_n);
    Vec prev(in_n, 0.0f);
    ref_backward_maxpool(out_n, delta.data(), idx.data(), prev.data());
    Dev dd(delta), dprev(in_n);
    g::backwardMaxpool(in_n, H, W, C, stride, size, pad, dd, dprev, didx);
    report("backward_maxpool", prev, pull(dprev, in_n), Exact);
    Vec avg(B * C);
    ref_forward_avgpool(B, C, H, W, x.data(), avg.data());
    Dev davg(B * C);
    g::forwardAvgpool(B * C, W, H, C, dx, davg);
    report("forward_avgpool", avg, pull(davg, B * C), Exact);
    const Vec od = random(rng, B * C);
    Vec ind = random(rng, in_n);
    Dev dind(ind), dod(od);
    ref_backward_avgpool(B, C, H, W, od.data(), ind.data());
    g::backwardAvgpool(B * C, W, H, C, dind, dod);
    report("backward_avgpool", ind, pull(dind, in_n), Exact);
}

void shortcutOp() {
    const int64_t B = 2, W = 8, H = 8, C = 4, n = B * W * H * C;
    Rng rng(20240925);
    const Vec add = random(rng, n), out = random(rng, n);
    Vec cpu = out;
    ref_shortcut(B, W, H, C, add.data(), W, H, C, 1.0f, 1.0f, cpu.data());
    Dev da(add), dout(out);
    g::shortcut(B, W, H, C, da, W, H, C, 1.0f, 1.0f, dout);
    report("shortcut", cpu, pull(dout, n), Exact);
}

void fusedEntries() {
    // batchnorm.zig:74-123 + activate, on [8, 16, 64] (the persistent kernel) and [4, 17, 53]
    // (the generic path); the per-element outputs must equal the reference sequence given the
    // device's own statistics, the statistics within the tolerance bar.
    const int64_t shapes[2][3] = {{8, 16, 64}, {4, 17, 53}};
    for (const auto &sh : shapes) {
        const int64_t B = sh[0], C = sh[1], S = sh[2], n = B * C * S;
        Rng rng(20240926 + C);
        const Vec x = random(rng, n, -2, 2), delta = random(rng, n), gamma = random(rng, C, 0.5f, 1.5f),
                  beta = random(rng, C, -0.1f, 0.1f);
        Dev dx(x), dy(n), dmean(C), dvar(C), drm(C), drv(C), dg(gamma), db(beta);
        g::bnActForwardTrain(dx, dy, g::Buf{}, B, C, S, dg, db, dmean, dvar, drm, drv, g::leaky);
        const Vec m = pull(dmean, C), v = pull(dvar, C);
        Vec rm(C, 0.0f), rv(C, 0.0f), mc(C), vc(C), y(n), xs(n), xn(n);
        ref_bn_forward_layer(x.data(), y.data(), xs.data(), xn.data(), B, C, S, gamma.data(), beta.data(), mc.data(),
                             vc.data(), rm.data(), rv.data(), 1, g::leaky);
        Vec sc = channel_norm(x, B, C, S);
        for (auto &t : sc) t /= (float)(B * S);
        const std::string tag = std::to_string(B) + "x" + std::to_string(C) + "x" + std::to_string(S);
        report(("bn_act_forward_train mean " + tag).c_str(), mc, m, Tol, &sc);
        // outputs given the device's statistics: normalize, scale, bias, activate
        Vec yw = x;
        ref_normalize(yw.data(), m.data(), v.data(), B, C, S);
        ref_scale_bias(yw.data(), gamma.data(), B, C, S);
        ref_add_bias(yw.data(), beta.data(), B, C, S);
        ref_activate_array(yw.data(), n, g::leaky);
        report(("bn_act_forward_train y " + tag).c_str(), yw, pull(dy, n), Exact);
        // backward with the device's statistics and its own mean_delta / variance_delta
        Dev dd(delta), ddx(n), dbu(C), dsu(C), dmd(C), dvd(C);
        g::bnActBackward(dx, g::Buf{}, dd, ddx, B, C, S, dg, db, dmean, dvar, dbu, dsu, dmd, dvd, g::leaky);
        const Vec md = pull(dmd, C), vd = pull(dvd, C);
        Vec gr = delta;
        ref_gradient_array(yw.data(), n, g::leaky, gr.data());
        ref_scale_bias(gr.data(), gamma.data(), B, C, S);
        Vec dxw = gr;
        ref_normalize_delta(x.data(), m.data(), v.data(), md.data(), vd.data(), B, C, S, dxw.data());
        report(("bn_act_backward dx " + tag).c_str(), dxw, pull(ddx, n), Exact);
    }
    {  // SGD with momentum: convolutional.zig:324-334
        const size_t n = 4099;
        Rng rng(20240927);
        Vec w = random(rng, n), wu = random(rng, n, -0.01f, 0.01f);
        Dev dw(w), dwu(wu);
        g::sgdMomentum(n, dw, dwu, 0.1f, 0.9f, 5e-4f, 64);
        ref_sgd_update(w.data(), wu.data(), n, 0.1f, 0.9f, 5e-4f, 64);
        report("sgd_momentum weights", w, pull(dw, n), Exact);
        report("sgd_momentum updates", wu, pull(dwu, n), Exact);
    }
}

}  // namespace

int main(int argc, char **argv) {
    list_only = argc > 1 && std::strcmp(argv[1], "--list") == 0;
    const Check all[] = {{"elementwise", elementwise}, {"biasAndNorm", biasAndNorm},
                         {"softmaxAndLoss", softmaxAndLoss}, {"pooling", pooling},
                         {"shortcutOp", shortcutOp}, {"fusedEntries", fusedEntries}};
    if (list_only) {
        for (const auto &c : all) std::printf("%s\n", c.section);
        return 0;
    }
    try {
        g::init(0);
        // synchronise after every launch: a fault is reported against the op that caused it
        // (gputest.zig:62-68)
        g::setSyncAfterLaunch(true);
        std::printf("\nComparing CPU and B200 implementations:\n\n");
        for (const auto &c : all) c.run();
        g::setSyncAfterLaunch(false);
    } catch (const std::exception &e) {
        std::printf("gputest: %s\n", e.what());
        return 2;
    }
    std::printf("\n%d/%d checks passed.\n", checks - failures, checks);
    return failures ? 1 : 0;
}
