// Fused batchnorm + activation, training forward and backward.
//
// The reference runs BN forward as copy -> mean -> variance -> 4 x C-vector EMA ops ->
// normalize -> copy(x_norm) -> scale_bias -> add_bias, then activate
// (batchnorm.zig:129-152, convolutional.zig:269): about 56 bytes of HBM traffic per
// element. Its backward (convolutional.zig:280, batchnorm.zig:155-169) is gradient ->
// backward_bias -> backward_scale -> scale_bias -> mean_delta -> variance_delta ->
// normalize_delta: about 56 bytes per element again. The compulsory traffic is 8 B/elem
// forward (read x, write y) and 12 B/elem backward (read delta and x, write dx).
//
// The obstacle is the per-channel reduction that must finish before any element can be
// written. The persistent kernel here removes the second read:
//   * one CTA per SM (cooperative launch, so every CTA is resident) owns ~200 KB of shared
//     memory split into two stage buffers;
//   * channels are processed in groups sized so that a group's units (contiguous runs of a
//     plane) fill every CTA's stage buffer once;
//   * a CTA pulls its share of group g into shared memory with 1-D bulk TMA copies,
//     reduces it per channel, publishes one partial record per (CTA, channel), and
//     arrives on a per-group counter in global memory;
//   * once all CTAs have arrived it merges the channel's records (Chan's parallel
//     variance formula, fp64), and writes the group's outputs straight from shared memory.
//     The copy of group g+1 is in flight during that wait, so HBM stays busy.
// Every wait is bounded: a CTA that gives up sets the device error word, waits (bounded)
// for its own copies, and exits; the host reports DNB_ERR_TIMEOUT.
//
// Shapes the persistent kernel does not take (spatial % 4 != 0, a channel larger than the
// whole grid's shared memory, unaligned pointers) run the generic three-launch path below,
// which also implements the split sync-BN entry points: per-channel partials ->
// (caller's collective) -> finalize + apply.
//
// Per-element arithmetic follows the reference CPU code (blas.zig:137-204) operation by
// operation without fused roundings (--fmad=false), so given the same per-channel
// statistics the outputs are bit-identical to it.
#include <math.h>

#include <cooperative_groups.h>

#include "dnb_chan.cuh"

namespace dnb {
namespace {

// ======================================================================================
// per-channel closing formulas shared by both paths
// ======================================================================================

// Forward: statistics -> outputs and the per-channel apply record.
// mean/var rounding: the reference computes sum*(1/n) and sum*(1/(n-1)) in f32
// (blas.zig:107,122); here the fp64 merge result is rounded once.
struct FwdClose {
    float m, var, inv;
};
__device__ __forceinline__ FwdClose fwd_close(double mean, double m2, double count) {
    FwdClose r;
    r.m = (float)mean;
    r.var = (float)(m2 / (count - 1.0));
    r.inv = 1.0f / (sqrtf(r.var) + 0.000001f);  // blas.zig:142
    return r;
}
// batchnorm.zig:140-143: scal(0.99) then axpy(1-0.99) with one fused rounding
__device__ __forceinline__ float rolling(float r, float stat) { return __fmaf_rn(1.0f - 0.99f, stat, r * 0.99f); }

struct BwdParam {
    float m, inv, g, b;       // forward normalisation (to recompute y) and scale/bias
    float inv2, vd, mdd, pad;  // normalize_delta terms: 1/sqrt(v+1e-5), variance_delta, mean_delta/denom
};

// Backward closing: s1 = sum(g), s2 = sum(g*(x-m)) over the whole (global) channel.
__device__ __forceinline__ BwdParam bwd_close(double s1, double s2, float m, float var, float gamma, float beta,
                                              float denom, float *bias_upd, float *scale_upd, float *mean_delta,
                                              float *var_delta, int64_t c, bool write) {
    BwdParam p;
    p.m = m;
    p.inv = 1.0f / (sqrtf(var) + 0.000001f);
    p.g = gamma;
    p.b = beta;
    p.inv2 = 1.0f / sqrtf(var + 0.00001f);                                               // blas.zig:195
    const float md = (float)((double)gamma * s1) * (-1.0f / sqrtf(var + 0.00001f));      // blas.zig:155
    const float vd = (float)((double)gamma * s2) * -0.5f * powf(var + 0.00001f, -1.5f);  // blas.zig:176
    p.vd = vd;
    p.mdd = md / denom;
    p.pad = 0.0f;
    if (write) {
        bias_upd[c] += (float)s1;                 // blas.zig:79
        scale_upd[c] += (float)(s2 * (double)p.inv);  // sum(g * x_norm), blas.zig:98
        mean_delta[c] = md;
        var_delta[c] = vd;
    }
    return p;
}

// y = act(((x - m) * inv) * gamma + beta): normalize, scaleBias, addBias, activate
template <int A>
__device__ __forceinline__ float bn_fwd1(float x, float m, float inv, float g, float b, int act) {
    return act_fwd<A>((x - m) * inv * g + b, act);
}
// g = delta * act'(y); y from the given output or recomputed from x
template <int A, bool HASY>
__device__ __forceinline__ float bn_grad1(float d, float x, float y, const BwdParam &p, int act) {
    const float yy = HASY ? y : bn_fwd1<A>(x, p.m, p.inv, p.g, p.b, act);
    return d * act_grad<A>(yy, act);
}
// dx = (g*gamma)*inv2 + vd*2*(x-m)/denom + md/denom (blas.zig:200 on delta*scales)
__device__ __forceinline__ float bn_dx1(float gval, float x, const BwdParam &p, float denom) {
    return (gval * p.g) * p.inv2 + p.vd * 2.0f * (x - p.m) / denom + p.mdd;
}

// ======================================================================================
// generic path: partials (grid of chunk x channel) -> close -> apply
// ======================================================================================

constexpr int kGThreads = 256;
constexpr int64_t kGChunk = 32768;

struct GGeom {
    int64_t batch, filters, spatial, per_channel, chunk;
    int chunks;
    bool vec, fast;
    FastDiv fs, fs4;
};

inline GGeom make_ggeom(int64_t batch, int64_t filters, int64_t spatial, bool aligned) {
    GGeom g;
    g.batch = batch;
    g.filters = filters;
    g.spatial = spatial;
    g.per_channel = batch * spatial;
    g.vec = spatial % 4 == 0 && aligned;
    g.chunk = kGChunk;
    int64_t chunks = (g.per_channel + g.chunk - 1) / g.chunk;
    g.chunks = (int)(chunks < 1 ? 1 : chunks);
    g.fast = g.per_channel < (1ll << 32);
    g.fs = FastDiv((uint32_t)(g.fast && spatial > 0 ? spatial : 1));
    g.fs4 = FastDiv((uint32_t)(g.fast && g.vec ? spatial / 4 : 1));
    return g;
}

// Visits this block's chunk of channel c: f(offset, count) for runs of 4 (vec) or 1.
template <class F>
__device__ __forceinline__ void for_chunk(const GGeom &g, int64_t c, F &&f) {
    const int64_t k0 = (int64_t)blockIdx.x * g.chunk;
    int64_t k1 = k0 + g.chunk;
    if (k1 > g.per_channel) k1 = g.per_channel;
    const int64_t cs = g.filters * g.spatial;
    if (g.vec) {
        const int64_t s4 = g.spatial >> 2;
        for (int64_t k = (k0 >> 2) + threadIdx.x; k < (k1 >> 2); k += kGThreads) {
            int64_t n, r;
            if (g.fast) {
                uint32_t q, rr;
                g.fs4.divmod((uint32_t)k, q, rr);
                n = q;
                r = rr;
            } else {
                n = k / s4;
                r = k - n * s4;
            }
            f(n * cs + c * g.spatial + 4 * r, 4);
        }
    } else {
        for (int64_t k = k0 + threadIdx.x; k < k1; k += kGThreads) {
            int64_t n, r;
            if (g.fast) {
                uint32_t q, rr;
                g.fs.divmod((uint32_t)k, q, rr);
                n = q;
                r = rr;
            } else {
                n = k / g.spatial;
                r = k - n * g.spatial;
            }
            f(n * cs + c * g.spatial + r, 1);
        }
    }
}

// Forward partial: shifted sums sum(x - shift), sum((x - shift)^2); shift = the channel's
// first element, so the one-pass form does not cancel for data whose mean is far from 0.
__global__ void __launch_bounds__(kGThreads) k_fwd_partial(GGeom g, const float *x, float2 *part) {
    __shared__ float red[64];
    const int64_t c = blockIdx.y;
    const float shift = x[c * g.spatial];
    float s1 = 0.0f, s2 = 0.0f;
    for_chunk(g, c, [&](int64_t off, int cnt) {
        if (cnt == 4) {
            const float4 v = ld4(x + off);
            const float a = v.x - shift, b = v.y - shift, cc = v.z - shift, d = v.w - shift;
            s1 += (a + b) + (cc + d);
            s2 += (a * a + b * b) + (cc * cc + d * d);
        } else {
            const float a = x[off] - shift;
            s1 += a;
            s2 += a * a;
        }
    });
    const float2 t = block_sum2<kGThreads>(s1, s2, red);
    if (threadIdx.x == 0) part[c * g.chunks + blockIdx.x] = t;
}

// Forward close: one thread per channel -> (mean, M2) of this rank's shard, fp64.
__global__ void k_fwd_local(GGeom g, const float *x, const float2 *part, double2 *local) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= g.filters) return;
    const double shift = x[c * g.spatial];
    double s1 = 0.0, s2 = 0.0;
    for (int i = 0; i < g.chunks; ++i) {
        const float2 t = part[c * g.chunks + i];
        s1 += t.x;
        s2 += t.y;
    }
    const double n = (double)g.per_channel;
    double m2 = s2 - s1 * s1 / n;
    if (m2 < 0.0) m2 = 0.0;
    local[c] = make_double2(shift + s1 / n, m2);
}

// Forward finalize over `ranks` equal-count records [rank][filters] -> outputs + table.
__global__ void k_fwd_finalize(int64_t filters, int ranks, double count_per_rank, const double2 *rec,
                               const float *scales, const float *biases, float *mean, float *var, float *rmean,
                               float *rvar, float4 *tab) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= filters) return;
    double msum = 0.0;
    for (int r = 0; r < ranks; ++r) msum += rec[(int64_t)r * filters + c].x;
    const double mu = msum / ranks;
    double m2 = 0.0;
    for (int r = 0; r < ranks; ++r) {
        const double2 t = rec[(int64_t)r * filters + c];
        const double d = t.x - mu;
        m2 += t.y + count_per_rank * d * d;
    }
    const FwdClose f = fwd_close(mu, m2, count_per_rank * ranks);
    mean[c] = f.m;
    var[c] = f.var;
    rmean[c] = rolling(rmean[c], f.m);
    rvar[c] = rolling(rvar[c], f.var);
    tab[c] = make_float4(f.m, f.inv, scales[c], biases[c]);
}

template <int A>
struct OpFwdApply {
    const float *x;
    float *y, *xn;
    const float4 *tab;
    int act;
    bool vec;
    using P = float4;
    using V = float4;
    __device__ P param(int64_t c) const { return tab[c]; }
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ static float f(float v, const P &p, int act) { return bn_fwd1<A>(v, p.x, p.y, p.z, p.w, act); }
    __device__ static float nrm(float v, const P &p) { return (v - p.x) * p.y; }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        if (xn) st4(xn + 4 * i, make_float4(nrm(v.x, p0), nrm(v.y, p1), nrm(v.z, p2), nrm(v.w, p3)));
        st4(y + 4 * i, make_float4(f(v.x, p0, act), f(v.y, p1, act), f(v.z, p2, act), f(v.w, p3, act)));
    }
    __device__ void scalar(int64_t i, P p) const {
        const float v = x[i];
        if (xn) xn[i] = nrm(v, p);
        y[i] = f(v, p, act);
    }
};

// Backward partial: s1 = sum(g), s2 = sum(g*(x-m)).
template <int A, bool HASY>
__global__ void __launch_bounds__(kGThreads) k_bwd_partial(GGeom g, const float *x, const float *y,
                                                         const float *delta, const float *mean, const float *var,
                                                         const float *scales, const float *biases, int act,
                                                         float2 *part) {
    __shared__ float red[64];
    const int64_t c = blockIdx.y;
    BwdParam p;
    p.m = mean[c];
    p.inv = 1.0f / (sqrtf(var[c]) + 0.000001f);
    p.g = scales[c];
    p.b = biases[c];
    float s1 = 0.0f, s2 = 0.0f;
    for_chunk(g, c, [&](int64_t off, int cnt) {
        if (cnt == 4) {
            const float4 d = ld4(delta + off), xv = ld4(x + off);
            const float4 yv = HASY ? ld4(y + off) : xv;
            const float g0 = bn_grad1<A, HASY>(d.x, xv.x, yv.x, p, act);
            const float g1 = bn_grad1<A, HASY>(d.y, xv.y, yv.y, p, act);
            const float g2 = bn_grad1<A, HASY>(d.z, xv.z, yv.z, p, act);
            const float g3 = bn_grad1<A, HASY>(d.w, xv.w, yv.w, p, act);
            s1 += (g0 + g1) + (g2 + g3);
            s2 += (g0 * (xv.x - p.m) + g1 * (xv.y - p.m)) + (g2 * (xv.z - p.m) + g3 * (xv.w - p.m));
        } else {
            const float gv = bn_grad1<A, HASY>(delta[off], x[off], HASY ? y[off] : 0.0f, p, act);
            s1 += gv;
            s2 += gv * (x[off] - p.m);
        }
    });
    const float2 t = block_sum2<kGThreads>(s1, s2, red);
    if (threadIdx.x == 0) part[c * g.chunks + blockIdx.x] = t;
}

__global__ void k_bwd_local(int64_t filters, int chunks, const float2 *part, double2 *local) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= filters) return;
    double s1 = 0.0, s2 = 0.0;
    for (int i = 0; i < chunks; ++i) {
        const float2 t = part[c * chunks + i];
        s1 += t.x;
        s2 += t.y;
    }
    local[c] = make_double2(s1, s2);
}

__global__ void k_bwd_finalize(int64_t filters, float denom, const double2 *sums, const float *mean, const float *var,
                               const float *scales, const float *biases, float *bias_upd, float *scale_upd,
                               float *mean_delta, float *var_delta, BwdParam *tab) {
    const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= filters) return;
    const double2 s = sums[c];
    tab[c] = bwd_close(s.x, s.y, mean[c], var[c], scales[c], biases[c], denom, bias_upd, scale_upd, mean_delta,
                       var_delta, c, true);
}

template <int A, bool HASY>
struct OpBwdApply {
    const float *x, *y, *d;
    float *dx;
    const BwdParam *tab;
    float denom;
    int act;
    bool vec;
    using P = BwdParam;
    struct V { float4 d, x, y; };
    __device__ P param(int64_t c) const { return tab[c]; }
    __device__ V load(int64_t i) const {
        V v;
        v.d = ld4(d + 4 * i);
        v.x = ld4(x + 4 * i);
        if (HASY) v.y = ld4(y + 4 * i);
        return v;
    }
    __device__ float f(float dv, float xv, float yv, const P &p) const {
        return bn_dx1(bn_grad1<A, HASY>(dv, xv, yv, p, act), xv, p, denom);
    }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        st4(dx + 4 * i, make_float4(f(v.d.x, v.x.x, v.y.x, p0), f(v.d.y, v.x.y, v.y.y, p1),
                                    f(v.d.z, v.x.z, v.y.z, p2), f(v.d.w, v.x.w, v.y.w, p3)));
    }
    __device__ void scalar(int64_t i, P p) const { dx[i] = f(d[i], x[i], HASY ? y[i] : 0.0f, p); }
};

// Scratch layout of the generic path inside the workspace.
struct GScratch {
    float2 *part;
    double2 *local;
    void *tab;
    static size_t bytes(const GGeom &g) {
        return align(sizeof(float2) * (size_t)(g.filters * g.chunks)) + align(sizeof(double2) * (size_t)g.filters) +
               align(sizeof(BwdParam) * (size_t)g.filters);
    }
    static size_t align(size_t b) { return (b + 255) & ~(size_t)255; }
    static GScratch carve(void *base, const GGeom &g) {
        GScratch s;
        char *p = static_cast<char *>(base);
        s.part = reinterpret_cast<float2 *>(p);
        p += align(sizeof(float2) * (size_t)(g.filters * g.chunks));
        s.local = reinterpret_cast<double2 *>(p);
        p += align(sizeof(double2) * (size_t)g.filters);
        s.tab = p;
        return s;
    }
};

dnb_status check_shape(int64_t batch, int64_t filters, int64_t spatial, const char *what) {
    if (batch < 0 || filters < 0 || spatial < 0) return fail(DNB_ERR_INVALID, "%s: negative size", what);
    if (filters > 65535) return fail(DNB_ERR_UNSUPPORTED, "%s: more than 65535 channels", what);
    if (filters > 0 && batch * spatial < 2)
        return fail(DNB_ERR_INVALID, "%s: batch*spatial must be >= 2 for the unbiased variance", what);
    return DNB_OK;
}

dnb_status generic_fwd_partials(const GGeom &g, const float *x, const GScratch &sc, cudaStream_t s) {
    k_fwd_partial<<<dim3((unsigned)g.chunks, (unsigned)g.filters), kGThreads, 0, s>>>(g, x, sc.part);
    DNB_TRY(after_launch(s, "bn forward partials"));
    k_fwd_local<<<(unsigned)((g.filters + 127) / 128), 128, 0, s>>>(g, x, sc.part, sc.local);
    return after_launch(s, "bn forward partials");
}

dnb_status generic_fwd_apply(const GGeom &g, const float *x, float *y, float *x_norm, const double2 *rec, int ranks,
                             const float *scales, const float *biases, float *mean, float *var, float *rmean,
                             float *rvar, int act, const GScratch &sc, cudaStream_t s) {
    float4 *tab = static_cast<float4 *>(sc.tab);
    k_fwd_finalize<<<(unsigned)((g.filters + 127) / 128), 128, 0, s>>>(
        g.filters, ranks, (double)g.per_channel, rec, scales, biases, mean, var, rmean, rvar, tab);
    DNB_TRY(after_launch(s, "bn forward finalize"));
    const bool al = aligned16(x) && aligned16(y) && (!x_norm || aligned16(x_norm));
    return dispatch_act(act, [&]<int A>() {
        return chan::launch_chan(g.batch, g.filters, g.spatial, OpFwdApply<A>{x, y, x_norm, tab, act, al}, s,
                                 "bn forward apply");
    });
}

dnb_status generic_bwd_partials(const GGeom &g, const float *x, const float *y, const float *delta, const float *mean,
                                const float *var, const float *scales, const float *biases, int act,
                                const GScratch &sc, cudaStream_t s) {
    const dim3 grid((unsigned)g.chunks, (unsigned)g.filters);
    DNB_TRY(dispatch_act(act, [&]<int A>() {
        if (y)
            k_bwd_partial<A, true><<<grid, kGThreads, 0, s>>>(g, x, y, delta, mean, var, scales, biases, act, sc.part);
        else
            k_bwd_partial<A, false><<<grid, kGThreads, 0, s>>>(g, x, y, delta, mean, var, scales, biases, act, sc.part);
        return after_launch(s, "bn backward partials");
    }));
    k_bwd_local<<<(unsigned)((g.filters + 127) / 128), 128, 0, s>>>(g.filters, g.chunks, sc.part, sc.local);
    return after_launch(s, "bn backward partials");
}

dnb_status generic_bwd_apply(const GGeom &g, const float *x, const float *y, const float *delta, float *dx,
                             float denom, const double2 *sums, const float *scales, const float *biases,
                             const float *mean, const float *var, float *bias_upd, float *scale_upd, float *mean_delta,
                             float *var_delta, int act, const GScratch &sc, cudaStream_t s) {
    BwdParam *tab = static_cast<BwdParam *>(sc.tab);
    k_bwd_finalize<<<(unsigned)((g.filters + 127) / 128), 128, 0, s>>>(
        g.filters, denom, sums, mean, var, scales, biases, bias_upd, scale_upd, mean_delta, var_delta, tab);
    DNB_TRY(after_launch(s, "bn backward finalize"));
    const bool al = aligned16(x) && aligned16(delta) && aligned16(dx) && (!y || aligned16(y));
    return dispatch_act(act, [&]<int A>() {
        if (y)
            return chan::launch_chan(g.batch, g.filters, g.spatial,
                                     OpBwdApply<A, true>{x, y, delta, dx, tab, denom, act, al}, s, "bn backward apply");
        return chan::launch_chan(g.batch, g.filters, g.spatial,
                                 OpBwdApply<A, false>{x, y, delta, dx, tab, denom, act, al}, s, "bn backward apply");
    });
}

// ======================================================================================
// persistent fused kernel
// ======================================================================================

constexpr int kPThreads = 256;
constexpr int kPMinBlocks = 2;  // CTAs per SM the register budget is sized for
constexpr int kMaxStages = 3;

__device__ __forceinline__ uint32_t smem_u32(const void *p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, unsigned parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// 1-D bulk copy global -> this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, unsigned bytes, uint64_t *bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

// Everything the persistent kernel needs, by value. All partition arithmetic is 32-bit
// with FastDiv: the plan guarantees cap_units * P * P < 2^32, which bounds every product
// below (p*T, (t+1)*P with T <= cap_units*P).
struct PArgs {
    // geometry
    int64_t C, S;
    int N, K, U, NK;       // batch, units per plane, unit floats, units per channel
    int cg, G, P;          // channels per group, groups, CTAs
    int cap_units, maxj, stages;
    uint32_t T_full, T_last;  // units in a group (every group but the last / the last)
    FastDiv f_u4, f_nk, f_k, f_p, f_tfull, f_tlast;
    float denom;           // batch*spatial as f32 (normalize_delta's denominator)
    float inv_denom;       // 1/denom, used only when denom is a power of two (then exact)
    int denom_pow2;
    // tensors: fwd uses t0 = x; bwd uses t0 = delta, t1 = x, t2 = y (optional)
    const float *t0, *t1, *t2;
    float *out, *xnorm;
    // per-channel parameters and outputs
    const float *scales, *biases;
    float *mean, *var, *rmean, *rvar;
    const float *mean_in, *var_in;
    float *bias_upd, *scale_upd, *mean_delta, *var_delta;
    int act;
    // workspace
    float2 *rec;           // [G][P][maxj]
    unsigned *sync;        // [0] epoch, then 2 banks of kMaxGroups counters
    unsigned *err, *abort_flag;
    unsigned long long wait_ns;
};

struct UnitEntry {
    long long goff;  // element offset of the unit in the tensors
    int j;           // channel slot within the CTA's share
    int pad;
};

// Share of CTA p in group g: units [t0, t1) of the group's T (channel base c0).
struct Share {
    uint32_t c0, T, t0, t1;
    int cfirst, clast;  // local channel indices touched (inclusive); cfirst > clast when empty
};
__device__ __forceinline__ Share share_of(const PArgs &a, int g, int p) {
    Share s;
    s.c0 = (uint32_t)g * (uint32_t)a.cg;
    s.T = g == a.G - 1 ? a.T_last : a.T_full;
    s.t0 = a.f_p.div((uint32_t)p * s.T);
    s.t1 = a.f_p.div((uint32_t)(p + 1) * s.T);
    s.cfirst = (int)a.f_nk.div(s.t0);
    s.clast = s.t1 > s.t0 ? (int)a.f_nk.div(s.t1 - 1) : s.cfirst - 1;
    return s;
}
// The CTA that owns unit t of group g: the largest p with floor(p*T/P) <= t.
__device__ __forceinline__ int owner_of(const PArgs &a, int g, uint32_t t) {
    const FastDiv &fd = g == a.G - 1 ? a.f_tlast : a.f_tfull;
    return (int)fd.div((t + 1) * (uint32_t)a.P - 1);
}

__device__ __forceinline__ float div_denom(float v, const PArgs &a) {
    return a.denom_pow2 ? v * a.inv_denom : v / a.denom;
}
// dx as bn_dx1, with the division by a power-of-two denominator done as an exact multiply
__device__ __forceinline__ float bn_dx_p(float gval, float x, const BwdParam &p, const PArgs &a) {
    return (gval * p.g) * p.inv2 + div_denom(p.vd * 2.0f * (x - p.m), a) + p.mdd;
}

template <bool BWD, int A, bool HASY>
struct PKernel {
    static constexpr int NT = BWD ? (HASY ? 3 : 2) : 1;  // tensors staged per unit

    struct Smem {
        float *buf;          // [stages][NT][cap_units*U]
        uint64_t *bars;      // [stages]
        UnitEntry *units;    // [stages][cap_units]
        float *ptab;         // apply records of the current group: [maxj][8]
        float *red;          // 64 floats
        int *flag;
    };

    // Byte offsets of the regions of dynamic shared memory, each 16-byte aligned.
    struct Layout {
        size_t bars, units, ptab, red, flag, total;
    };
    __host__ __device__ static size_t up16(size_t b) { return (b + 15) & ~(size_t)15; }
    __host__ __device__ static Layout layout(int stages, int cap_units, int U, int maxj) {
        Layout l;
        l.bars = up16((size_t)stages * NT * cap_units * U * sizeof(float));
        l.units = up16(l.bars + kMaxStages * sizeof(uint64_t));
        l.ptab = up16(l.units + (size_t)stages * cap_units * sizeof(UnitEntry));
        l.red = up16(l.ptab + (size_t)maxj * 8 * sizeof(float));
        l.flag = up16(l.red + 64 * sizeof(float));
        l.total = l.flag + 16;
        return l;
    }
    __device__ static Smem carve(const PArgs &a, unsigned char *raw) {
        const Layout l = layout(a.stages, a.cap_units, a.U, a.maxj);
        Smem s;
        s.buf = reinterpret_cast<float *>(raw);
        s.bars = reinterpret_cast<uint64_t *>(raw + l.bars);
        s.units = reinterpret_cast<UnitEntry *>(raw + l.units);
        s.ptab = reinterpret_cast<float *>(raw + l.ptab);
        s.red = reinterpret_cast<float *>(raw + l.red);
        s.flag = reinterpret_cast<int *>(raw + l.flag);
        return s;
    }
    __host__ static size_t smem_bytes(int stages, int cap_units, int U, int maxj) {
        return layout(stages, cap_units, U, maxj).total;
    }

    __device__ static float *tensor_buf(const PArgs &a, const Smem &s, int stage, int t) {
        return s.buf + ((size_t)stage * NT + t) * a.cap_units * a.U;
    }

    // Issue the copies of group g into `stage` (warp 0; lane 0 arms the barrier first).
    __device__ static void issue(const PArgs &a, const Smem &s, int g, int stage) {
        if (threadIdx.x >= 32) return;
        const Share sh = share_of(a, g, blockIdx.x);
        const int n_units = (int)(sh.t1 - sh.t0);
        const unsigned unit_bytes = (unsigned)a.U * sizeof(float);
        if (threadIdx.x == 0) {
            fence_proxy_async();
            mbar_arrive_expect_tx(&s.bars[stage], (unsigned)(n_units * NT) * unit_bytes);
        }
        __syncwarp();
        const float *src[3] = {a.t0, a.t1, a.t2};
        for (int u = threadIdx.x; u < n_units; u += 32) {
            const uint32_t t = sh.t0 + u;
            uint32_t cl, rem, n, k;
            a.f_nk.divmod(t, cl, rem);
            a.f_k.divmod(rem, n, k);
            const int64_t c = (int64_t)sh.c0 + cl;
            const int64_t goff = ((int64_t)n * a.C + c) * a.S + (int64_t)k * a.U;
            s.units[stage * a.cap_units + u] = UnitEntry{goff, (int)cl - sh.cfirst, 0};
#pragma unroll
            for (int tt = 0; tt < NT; ++tt)
                bulk_g2s(tensor_buf(a, s, stage, tt) + (size_t)u * a.U, src[tt] + goff, unit_bytes, &s.bars[stage]);
        }
    }

    // Wait (bounded) for the copies of `stage` with the given phase parity.
    __device__ static bool wait_copies(const PArgs &a, const Smem &s, int stage, unsigned parity) {
        const unsigned long long deadline = global_ns() + a.wait_ns;
        unsigned it = 0;
        while (!mbar_try_wait(&s.bars[stage], parity)) {
            if ((++it & 63u) == 0 && global_ns() > deadline) {
                atomicOr(a.err, DEVERR_WAIT_COPY);
                atomicExch(a.abort_flag, 1u);
                return false;
            }
        }
        return true;
    }

    // Per-channel partial of one share segment (the whole block; result valid in thread 0).
    __device__ static float2 segment_stats(const PArgs &a, const Smem &s, int stage, int ua, int ub, int64_t c) {
        const int q0 = ua * (a.U >> 2), q1 = ub * (a.U >> 2);  // float4 range in the stage buffer
        const float4 *b0 = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, 0));
        if constexpr (!BWD) {
            // one pass: per-thread sums shifted by the thread's first element, then the block
            // merges (count, mean, M2) of its threads (Chan et al.)
            float shift = 0.0f, s1 = 0.0f, s2 = 0.0f, nt = 0.0f;
            if (q0 + (int)threadIdx.x < q1) shift = b0[q0 + threadIdx.x].x;
            for (int q = q0 + threadIdx.x; q < q1; q += kPThreads) {
                const float4 v = b0[q];
                const float d0 = v.x - shift, d1 = v.y - shift, d2 = v.z - shift, d3 = v.w - shift;
                s1 += (d0 + d1) + (d2 + d3);
                s2 += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
                nt += 4.0f;
            }
            const float cnt = (float)((q1 - q0) * 4);
            const float mt = nt > 0.0f ? shift + s1 / nt : 0.0f;
            float m2t = nt > 0.0f ? s2 - s1 * (s1 / nt) : 0.0f;
            if (m2t < 0.0f) m2t = 0.0f;
            const float mr = block_sum<kPThreads>(nt > 0.0f ? nt * shift + s1 : 0.0f, s.red) / cnt;
            const float dm = mt - mr;
            const float m2 = block_sum<kPThreads>(nt > 0.0f ? m2t + nt * dm * dm : 0.0f, s.red);
            return make_float2(mr, m2);
        } else {
            const float4 *bx = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, 1));
            const float4 *by = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, NT - 1));
            BwdParam p;
            p.m = a.mean_in[c];
            p.inv = 1.0f / (sqrtf(a.var_in[c]) + 0.000001f);
            p.g = a.scales[c];
            p.b = a.biases[c];
            float s1 = 0.0f, s2 = 0.0f;
            for (int q = q0 + threadIdx.x; q < q1; q += kPThreads) {
                const float4 d = b0[q], xv = bx[q];
                const float4 yv = HASY ? by[q] : xv;
                const float g0 = bn_grad1<A, HASY>(d.x, xv.x, yv.x, p, a.act);
                const float g1 = bn_grad1<A, HASY>(d.y, xv.y, yv.y, p, a.act);
                const float g2 = bn_grad1<A, HASY>(d.z, xv.z, yv.z, p, a.act);
                const float g3 = bn_grad1<A, HASY>(d.w, xv.w, yv.w, p, a.act);
                s1 += (g0 + g1) + (g2 + g3);
                s2 += (g0 * (xv.x - p.m) + g1 * (xv.y - p.m)) + (g2 * (xv.z - p.m) + g3 * (xv.w - p.m));
            }
            return block_sum2<kPThreads>(s1, s2, s.red);
        }
    }

    // Partials of every channel segment of this CTA's share of group g -> records.
    __device__ static void stats(const PArgs &a, const Smem &s, int g, int stage) {
        const Share sh = share_of(a, g, blockIdx.x);
        for (int cl = sh.cfirst; cl <= sh.clast; ++cl) {
            uint32_t ua = (uint32_t)cl * a.NK, ub = ua + a.NK;
            if (ua < sh.t0) ua = sh.t0;
            if (ub > sh.t1) ub = sh.t1;
            const float2 r = segment_stats(a, s, stage, (int)(ua - sh.t0), (int)(ub - sh.t0), (int64_t)sh.c0 + cl);
            if (threadIdx.x == 0)
                a.rec[((int64_t)g * a.P + blockIdx.x) * a.maxj + (cl - sh.cfirst)] = r;
        }
    }

    // Publish this CTA's records of group g: fence, then one arrival on the group counter.
    __device__ static void arrive(const PArgs &a, unsigned *cnt, int g, bool last_group, unsigned epoch) {
        if (threadIdx.x == 0) {
            __threadfence();
            const unsigned prev = atomicAdd(&cnt[g], 1u);
            // every CTA read the epoch before its first arrival: the last one of the last
            // group advances it for the next launch
            if (last_group && prev == (unsigned)a.P - 1) atomicExch(&a.sync[0], epoch + 1);
        }
    }

    // Wait (bounded) until every CTA has arrived on group g; block-uniform result.
    __device__ static bool wait_group(const PArgs &a, const Smem &s, unsigned *cnt, int g) {
        if (threadIdx.x == 0) {
            int ok = 1;
            const unsigned long long deadline = global_ns() + a.wait_ns;
            while (ld_acquire_gpu(&cnt[g]) < (unsigned)a.P) {
                if (ld_volatile(a.abort_flag)) {
                    ok = 0;
                    break;
                }
                if (global_ns() > deadline) {
                    atomicOr(a.err, DEVERR_WAIT_BARRIER);
                    atomicExch(a.abort_flag, 1u);
                    ok = 0;
                    break;
                }
                __nanosleep(32);
            }
            *s.flag = ok;
        }
        __syncthreads();
        return *s.flag != 0;
    }

    // Merge the records of every channel this CTA's share of group g touches and build the
    // apply table; the CTA owning a channel's first unit writes the per-channel outputs.
    __device__ static void finalize(const PArgs &a, const Smem &s, int g) {
        const Share sh = share_of(a, g, blockIdx.x);
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        for (int cl = sh.cfirst + warp; cl <= sh.clast; cl += kPThreads / 32) {
            const int64_t c = (int64_t)sh.c0 + cl;
            const uint32_t ua = (uint32_t)cl * a.NK, ub = ua + a.NK;
            const int plo = owner_of(a, g, ua), phi = owner_of(a, g, ub - 1);
            const bool write = plo == (int)blockIdx.x;
            float *out = s.ptab + (cl - sh.cfirst) * 8;
            // CTAs between plo and phi with no unit of this channel (a group with fewer
            // units than CTAs) wrote no record for it: skip them
            if constexpr (!BWD) {
                double cm = 0.0, n_r = 0.0, m_r = 0.0, q_r = 0.0;
                bool have = false;
                for (int p = plo + lane; p <= phi; p += 32) {
                    const Share o = share_of(a, g, p);
                    const uint32_t lo = ua > o.t0 ? ua : o.t0, hi = ub < o.t1 ? ub : o.t1;
                    if (hi <= lo) continue;
                    const float2 r = __ldcg(&a.rec[((int64_t)g * a.P + p) * a.maxj + (cl - o.cfirst)]);
                    const double nr = (double)((hi - lo) * (uint32_t)a.U);
                    cm += nr * (double)r.x;
                    if (p + 32 > phi) {  // the common case: one record per lane
                        n_r = nr;
                        m_r = r.x;
                        q_r = r.y;
                        have = true;
                    }
                }
                const double n = (double)a.NK * a.U;
                const double mu = warp_sum(cm) / n;
                double m2 = 0.0;
                if (phi - plo < 32) {
                    if (have) m2 = q_r + n_r * (m_r - mu) * (m_r - mu);
                } else {
                    for (int p = plo + lane; p <= phi; p += 32) {
                        const Share o = share_of(a, g, p);
                        const uint32_t lo = ua > o.t0 ? ua : o.t0, hi = ub < o.t1 ? ub : o.t1;
                        if (hi <= lo) continue;
                        const float2 r = __ldcg(&a.rec[((int64_t)g * a.P + p) * a.maxj + (cl - o.cfirst)]);
                        const double d = (double)r.x - mu;
                        m2 += (double)r.y + (double)((hi - lo) * (uint32_t)a.U) * d * d;
                    }
                }
                m2 = warp_sum(m2);
                if (lane == 0) {
                    const FwdClose f = fwd_close(mu, m2, n);
                    if (write) {
                        a.mean[c] = f.m;
                        a.var[c] = f.var;
                        a.rmean[c] = rolling(a.rmean[c], f.m);
                        a.rvar[c] = rolling(a.rvar[c], f.var);
                    }
                    out[0] = f.m;
                    out[1] = f.inv;
                    out[2] = a.scales[c];
                    out[3] = a.biases[c];
                }
            } else {
                double s1 = 0.0, s2 = 0.0;
                for (int p = plo + lane; p <= phi; p += 32) {
                    const Share o = share_of(a, g, p);
                    const uint32_t lo = ua > o.t0 ? ua : o.t0, hi = ub < o.t1 ? ub : o.t1;
                    if (hi <= lo) continue;
                    const float2 r = __ldcg(&a.rec[((int64_t)g * a.P + p) * a.maxj + (cl - o.cfirst)]);
                    s1 += (double)r.x;
                    s2 += (double)r.y;
                }
                s1 = warp_sum(s1);
                s2 = warp_sum(s2);
                if (lane == 0) {
                    const BwdParam bp = bwd_close(s1, s2, a.mean_in[c], a.var_in[c], a.scales[c], a.biases[c],
                                                  a.denom, a.bias_upd, a.scale_upd, a.mean_delta, a.var_delta, c,
                                                  write);
                    *reinterpret_cast<BwdParam *>(out) = bp;
                }
            }
        }
        __syncthreads();
    }

    __device__ static void apply(const PArgs &a, const Smem &s, int g, int stage) {
        const Share sh = share_of(a, g, blockIdx.x);
        const uint32_t u4 = (uint32_t)a.U >> 2;
        const uint32_t n4 = (sh.t1 - sh.t0) * u4;
        const float4 *b0 = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, 0));
        const UnitEntry *ut = s.units + stage * a.cap_units;
        if constexpr (!BWD) {
            for (uint32_t i = threadIdx.x; i < n4; i += kPThreads) {
                uint32_t u, r;
                a.f_u4.divmod(i, u, r);
                const UnitEntry e = ut[u];
                const float4 p = *reinterpret_cast<const float4 *>(s.ptab + e.j * 8);
                const float4 v = b0[i];
                const int64_t off = e.goff + 4 * (int64_t)r;
                if (a.xnorm)
                    st4(a.xnorm + off, make_float4((v.x - p.x) * p.y, (v.y - p.x) * p.y, (v.z - p.x) * p.y,
                                                   (v.w - p.x) * p.y));
                st4(a.out + off, make_float4(bn_fwd1<A>(v.x, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v.y, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v.z, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v.w, p.x, p.y, p.z, p.w, a.act)));
            }
        } else {
            const float4 *bx = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, 1));
            const float4 *by = reinterpret_cast<const float4 *>(tensor_buf(a, s, stage, NT - 1));
            for (uint32_t i = threadIdx.x; i < n4; i += kPThreads) {
                uint32_t u, r;
                a.f_u4.divmod(i, u, r);
                const UnitEntry e = ut[u];
                const BwdParam p = *reinterpret_cast<const BwdParam *>(s.ptab + e.j * 8);
                const float4 d = b0[i], xv = bx[i];
                const float4 yv = HASY ? by[i] : xv;
                const int64_t off = e.goff + 4 * (int64_t)r;
                st4(a.out + off, make_float4(bn_dx_p(bn_grad1<A, HASY>(d.x, xv.x, yv.x, p, a.act), xv.x, p, a),
                                             bn_dx_p(bn_grad1<A, HASY>(d.y, xv.y, yv.y, p, a.act), xv.y, p, a),
                                             bn_dx_p(bn_grad1<A, HASY>(d.z, xv.z, yv.z, p, a.act), xv.z, p, a),
                                             bn_dx_p(bn_grad1<A, HASY>(d.w, xv.w, yv.w, p, a.act), xv.w, p, a)));
            }
        }
    }
};

#ifdef DNB_PHASE_TIMING
// Diagnostic build only (-DDNB_PHASE_TIMING): %globaltimer stamps per (CTA, group, phase):
// 0 copies landed, 1 partials published, 2 group barrier released, 3 merge done, 4 apply done.
constexpr int kTsCtas = 160, kTsGroups = 64, kTsPhases = 6;
__device__ unsigned long long g_phase_ts[kTsCtas * kTsGroups * kTsPhases];
#define DNB_STAMP(g, ph)                                                                              \
    do {                                                                                              \
        if (threadIdx.x == 0 && blockIdx.x < kTsCtas && (g) < kTsGroups)                              \
            g_phase_ts[(blockIdx.x * kTsGroups + (g)) * kTsPhases + (ph)] = global_ns();              \
    } while (0)
#else
#define DNB_STAMP(g, ph) \
    do {                 \
    } while (0)
#endif

// Software pipeline, `stages` groups deep. Iteration g:
//   wait for group g+1's copies; reduce them; publish (arrive on g+1)
//   wait for group g's arrivals (published one iteration earlier, so normally complete)
//   merge group g's records; write group g's outputs from shared memory
//   refill the freed stage with group g+stages
// The copy of a group is issued `stages - 1` iterations before it is reduced, and the
// grid-wide wait for a group trails its arrivals by one iteration of work.
template <bool BWD, int A, bool HASY>
__global__ void __launch_bounds__(kPThreads, kPMinBlocks) k_bn_persistent(PArgs a) {
    using K = PKernel<BWD, A, HASY>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const typename K::Smem s = K::carve(a, smem_raw);
    __shared__ unsigned s_epoch;

    if (threadIdx.x == 0) {
        s_epoch = ld_volatile(&a.sync[0]);
        for (int i = 0; i < a.stages; ++i) mbar_init(&s.bars[i], 1);
        fence_mbar_init();
    }
    __syncthreads();
    const unsigned epoch = s_epoch;
    unsigned *cnt = a.sync + 1 + (epoch & 1u) * kMaxGroups;
    if (blockIdx.x == 0) {
        unsigned *other = a.sync + 1 + ((epoch & 1u) ^ 1u) * kMaxGroups;
        for (int i = threadIdx.x; i < kMaxGroups; i += kPThreads) other[i] = 0u;
    }

    // pending[st] = parity of the copy outstanding on stage st, or -1
    int pending[kMaxStages] = {-1, -1, -1};
    unsigned uses[kMaxStages] = {0, 0, 0};

    const int pre = a.G < a.stages ? a.G : a.stages;
    for (int g = 0; g < pre; ++g) {
        K::issue(a, s, g, g);
        pending[g] = (int)(uses[g] & 1u);
        ++uses[g];
    }
    // every wait result is made block-uniform before it steers control flow, so no thread
    // can leave the loop while others continue into a barrier
    bool ok = __syncthreads_and(K::wait_copies(a, s, 0, (unsigned)pending[0])) != 0;
    DNB_STAMP(0, 0);
    if (ok) {
        K::stats(a, s, 0, 0);
        K::arrive(a, cnt, 0, a.G == 1, epoch);
        DNB_STAMP(0, 1);
    }
    for (int g = 0; ok && g < a.G; ++g) {
        const int st = g % a.stages;
        if (g + 1 < a.G) {
            const int st1 = (g + 1) % a.stages;
            ok = __syncthreads_and(K::wait_copies(a, s, st1, (unsigned)pending[st1])) != 0;
            DNB_STAMP(g + 1, 0);
            if (!ok) break;
            K::stats(a, s, g + 1, st1);
            K::arrive(a, cnt, g + 1, g + 2 == a.G, epoch);
            DNB_STAMP(g + 1, 1);
        }
        ok = K::wait_group(a, s, cnt, g);
        DNB_STAMP(g, 2);
        if (!ok) break;
        K::finalize(a, s, g);
        DNB_STAMP(g, 3);
        K::apply(a, s, g, st);
        pending[st] = -1;
        __syncthreads();  // every thread is done reading stage st
        DNB_STAMP(g, 4);
        if (g + a.stages < a.G) {
            K::issue(a, s, g + a.stages, st);
            pending[st] = (int)(uses[st] & 1u);
            ++uses[st];
        }
    }
    if (!ok) {
        // leave no copy in flight into this CTA's shared memory
        for (int st = 0; st < a.stages; ++st)
            if (pending[st] >= 0) K::wait_copies(a, s, st, (unsigned)pending[st]);
    }
}

struct PPlan {
    bool ok = false;
    int K, U, cap_units, cg, G, P, maxj, stages, ctas_per_sm;
    size_t smem;
};

// Shapes the persistent kernel: units of U = spatial/K floats (U % 4 == 0), a stage
// buffer per tensor of cap_units units, cg channels per group.
template <bool BWD, bool HASY>
PPlan plan_persistent(int64_t batch, int64_t filters, int64_t spatial, const DeviceState *ds, int stages) {
    using K = PKernel<BWD, DNB_ACT_LEAKY, HASY>;
    PPlan pl;
    if (spatial % 4 != 0 || batch <= 0 || filters <= 0) return pl;
    const int nt = K::NT;
    // CTAs per SM: two by default, so one CTA's barrier wait and merge overlap the other's
    // reduction and writes
    const char *env_c = getenv("DNB_BN_CTAS_PER_SM");
    int ctas = env_c ? atoi(env_c) : 2;
    if (ctas < 1) ctas = 1;
    if (ctas > 4) ctas = 4;
    size_t per_cta = (size_t)ds->smem_per_sm / ctas - (size_t)ds->smem_reserved - 256;  // 256: static smem
    if (per_cta > (size_t)ds->max_smem_optin) per_cta = (size_t)ds->max_smem_optin;
    const size_t budget = per_cta - 4096;  // unit tables, apply records, reduction scratch, barriers
    const size_t per_tensor = budget / ((size_t)stages * nt);
    // smallest K dividing spatial with U % 4 == 0 and one unit fitting a stage buffer
    int64_t k = 1;
    for (; k <= spatial; ++k) {
        if (spatial % k) continue;
        const int64_t u = spatial / k;
        if (u % 4 == 0 && (size_t)u * 4 <= per_tensor) break;
    }
    if (k > spatial) return pl;
    const int64_t U = spatial / k, NK = batch * k;
    int64_t cap = (int64_t)(per_tensor / ((size_t)U * 4));
    const int64_t P = (int64_t)ds->sm_count * ctas;
    int64_t cg_max = cap * P / NK;
    if (cg_max < 1) return pl;
    // at least ~6 groups so the copy of the next group overlaps the current one
    const char *env = getenv("DNB_BN_MIN_GROUPS");
    const int64_t min_groups = env ? atoll(env) : 6;
    int64_t cg = cg_max;
    if (min_groups > 1) {
        const int64_t want = (filters + min_groups - 1) / min_groups;
        if (want < cg) cg = want < 1 ? 1 : want;
    }
    int64_t G = (filters + cg - 1) / cg;
    cg = (filters + G - 1) / G;
    G = (filters + cg - 1) / cg;
    if (G > kMaxGroups) return pl;
    const int64_t share = (cg * NK + P - 1) / P;
    if (share > cap) return pl;
    // 32-bit partition arithmetic: every product is at most T*P <= share*P*P
    if ((uint64_t)share * P * P >= (1ull << 32)) return pl;
    cap = share;  // stage buffers only as large as a share
    pl.K = (int)k;
    pl.U = (int)U;
    pl.cap_units = (int)cap;
    pl.cg = (int)cg;
    pl.G = (int)G;
    pl.P = (int)P;
    pl.maxj = (int)((cap - 1) / NK + 2);
    pl.stages = stages;
    pl.smem = K::smem_bytes(stages, pl.cap_units, pl.U, pl.maxj);
    pl.ok = pl.smem <= per_cta;
    pl.ctas_per_sm = ctas;
    return pl;
}

int stages_from_env() {
    const char *e = getenv("DNB_BN_STAGES");
    int s = e ? atoi(e) : 3;
    return s < 2 ? 2 : (s > kMaxStages ? kMaxStages : s);
}

bool persistent_disabled() {
    const char *e = getenv("DNB_BN_PERSISTENT");
    return e && e[0] == '0';
}

template <bool BWD, bool HASY>
dnb_status launch_persistent(const PPlan &pl, PArgs &a, int act, cudaStream_t stream, const char *what) {
    return dispatch_act(act, [&]<int A>() -> dnb_status {
        auto kern = k_bn_persistent<BWD, A, HASY>;
        DNB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)pl.smem));
        int per_sm = 0;
        DNB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kPThreads, pl.smem));
        if (per_sm < pl.ctas_per_sm)
            return fail(DNB_ERR_UNSUPPORTED, "%s: %d CTAs of the persistent kernel fit an SM, the plan needs %d",
                        what, per_sm, pl.ctas_per_sm);
        void *args[] = {&a};
        DNB_CUDA(cudaLaunchCooperativeKernel((const void *)kern, dim3((unsigned)pl.P), dim3(kPThreads), args, pl.smem,
                                             stream));
        return after_launch(stream, what);
    });
}

template <bool BWD, bool HASY>
dnb_status prepare_persistent(int64_t batch, int64_t filters, int64_t spatial, cudaStream_t stream, PPlan *pl_out,
                              PArgs *a) {
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const PPlan pl = plan_persistent<BWD, HASY>(batch, filters, spatial, ds, stages_from_env());
    *pl_out = pl;
    if (!pl.ok) return DNB_OK;
    Workspace *ws = nullptr;
    DNB_TRY(workspace(stream, sizeof(float2) * (size_t)pl.G * pl.P * pl.maxj, &ws));
    a->C = filters;
    a->S = spatial;
    a->N = (int)batch;
    a->K = pl.K;
    a->U = pl.U;
    a->NK = (int)(batch * pl.K);
    a->cg = pl.cg;
    a->G = pl.G;
    a->P = pl.P;
    a->cap_units = pl.cap_units;
    a->maxj = pl.maxj;
    a->stages = pl.stages;
    a->f_u4 = FastDiv((uint32_t)(pl.U / 4));
    a->f_nk = FastDiv((uint32_t)a->NK);
    a->f_k = FastDiv((uint32_t)pl.K);
    a->f_p = FastDiv((uint32_t)pl.P);
    a->T_full = (uint32_t)pl.cg * (uint32_t)a->NK;
    a->T_last = (uint32_t)(filters - (int64_t)(pl.G - 1) * pl.cg) * (uint32_t)a->NK;
    a->f_tfull = FastDiv(a->T_full);
    a->f_tlast = FastDiv(a->T_last);
    a->denom = (float)(spatial * batch);
    // dividing by a power of two equals multiplying by its exact reciprocal
    int e2 = 0;
    const float fr = frexpf(a->denom, &e2);
    a->denom_pow2 = fr == 0.5f;
    a->inv_denom = 1.0f / a->denom;
    a->rec = static_cast<float2 *>(ws->scratch);
    a->sync = ws->sync;
    a->err = ds->error_word;
    a->abort_flag = ds->abort_flag;
    a->wait_ns = wait_limit_ns();
    return DNB_OK;
}

}  // namespace
}  // namespace dnb

using namespace dnb;

#ifdef DNB_PHASE_TIMING
extern "C" dnb_status dnb_debug_phase_times(unsigned long long *host, size_t count) {
    DNB_CUDA(cudaDeviceSynchronize());
    DNB_CUDA(cudaMemcpyFromSymbol(host, g_phase_ts, count * sizeof(unsigned long long)));
    return DNB_OK;
}
#endif

extern "C" {

dnb_status dnb_bn_act_forward_train(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                    int64_t spatial, const float *scales, const float *biases, float *mean,
                                    float *variance, float *rolling_mean, float *rolling_variance, int act,
                                    dnb_stream stream) {
    const char *what = "bn_act_forward_train";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (filters == 0) return DNB_OK;
    if (!x || !y || !scales || !biases || !mean || !variance || !rolling_mean || !rolling_variance)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const bool al = aligned16(x) && aligned16(y) && (!x_norm || aligned16(x_norm));
    if (al && !persistent_disabled()) {
        PPlan pl;
        PArgs a{};
        DNB_TRY((prepare_persistent<false, false>(batch, filters, spatial, s, &pl, &a)));
        if (pl.ok) {
            a.t0 = x;
            a.out = y;
            a.xnorm = x_norm;
            a.scales = scales;
            a.biases = biases;
            a.mean = mean;
            a.var = variance;
            a.rmean = rolling_mean;
            a.rvar = rolling_variance;
            a.act = act;
            return launch_persistent<false, false>(pl, a, act, s, what);
        }
    }
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    DNB_TRY(generic_fwd_partials(g, x, sc, s));
    return generic_fwd_apply(g, x, y, x_norm, sc.local, 1, scales, biases, mean, variance, rolling_mean,
                             rolling_variance, act, sc, s);
}

dnb_status dnb_bn_act_backward(const float *x, const float *y, const float *delta, float *dx, int64_t batch,
                               int64_t filters, int64_t spatial, const float *scales, const float *biases,
                               const float *mean, const float *variance, float *bias_updates, float *scale_updates,
                               float *mean_delta, float *variance_delta, int act, dnb_stream stream) {
    const char *what = "bn_act_backward";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (filters == 0) return DNB_OK;
    if (!x || !delta || !dx || !scales || !biases || !mean || !variance || !bias_updates || !scale_updates ||
        !mean_delta || !variance_delta)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const bool al = aligned16(x) && aligned16(delta) && aligned16(dx) && (!y || aligned16(y));
    if (al && !persistent_disabled()) {
        PPlan pl;
        PArgs a{};
        if (y)
            DNB_TRY((prepare_persistent<true, true>(batch, filters, spatial, s, &pl, &a)));
        else
            DNB_TRY((prepare_persistent<true, false>(batch, filters, spatial, s, &pl, &a)));
        if (pl.ok) {
            a.t0 = delta;
            a.t1 = x;
            a.t2 = y;
            a.out = dx;
            a.scales = scales;
            a.biases = biases;
            a.mean_in = mean;
            a.var_in = variance;
            a.bias_upd = bias_updates;
            a.scale_upd = scale_updates;
            a.mean_delta = mean_delta;
            a.var_delta = variance_delta;
            a.act = act;
            return y ? launch_persistent<true, true>(pl, a, act, s, what)
                     : launch_persistent<true, false>(pl, a, act, s, what);
        }
    }
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x) && aligned16(delta) && (!y || aligned16(y)));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    DNB_TRY(generic_bwd_partials(g, x, y, delta, mean, variance, scales, biases, act, sc, s));
    return generic_bwd_apply(g, x, y, delta, dx, (float)(spatial * batch), sc.local, scales, biases, mean, variance,
                             bias_updates, scale_updates, mean_delta, variance_delta, act, sc, s);
}

dnb_status dnb_syncbn_forward_partials(const float *x, int64_t batch, int64_t filters, int64_t spatial,
                                       double *partials, dnb_stream stream) {
    const char *what = "syncbn_forward_partials";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (filters == 0) return DNB_OK;
    if (!x || !partials) return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    GScratch sc = GScratch::carve(ws->scratch, g);
    sc.local = reinterpret_cast<double2 *>(partials);
    return generic_fwd_partials(g, x, sc, s);
}

dnb_status dnb_syncbn_forward_apply(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                    int64_t spatial, const double *gathered, int ranks, const float *scales,
                                    const float *biases, float *mean, float *variance, float *rolling_mean,
                                    float *rolling_variance, int act, dnb_stream stream) {
    const char *what = "syncbn_forward_apply";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (ranks < 1) return fail(DNB_ERR_INVALID, "%s: ranks must be >= 1", what);
    if (filters == 0) return DNB_OK;
    if (!x || !y || !gathered || !scales || !biases || !mean || !variance || !rolling_mean || !rolling_variance)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    return generic_fwd_apply(g, x, y, x_norm, reinterpret_cast<const double2 *>(gathered), ranks, scales, biases, mean,
                             variance, rolling_mean, rolling_variance, act, sc, s);
}

dnb_status dnb_syncbn_backward_partials(const float *x, const float *y, const float *delta, int64_t batch,
                                        int64_t filters, int64_t spatial, const float *scales, const float *biases,
                                        const float *mean, const float *variance, int act, double *partials,
                                        dnb_stream stream) {
    const char *what = "syncbn_backward_partials";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (filters == 0) return DNB_OK;
    if (!x || !delta || !scales || !biases || !mean || !variance || !partials)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x) && aligned16(delta) && (!y || aligned16(y)));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    GScratch sc = GScratch::carve(ws->scratch, g);
    sc.local = reinterpret_cast<double2 *>(partials);
    return generic_bwd_partials(g, x, y, delta, mean, variance, scales, biases, act, sc, s);
}

dnb_status dnb_syncbn_backward_apply(const float *x, const float *y, const float *delta, float *dx, int64_t batch,
                                     int64_t filters, int64_t spatial, int64_t total_count, const double *reduced,
                                     const float *scales, const float *biases, const float *mean,
                                     const float *variance, float *bias_updates, float *scale_updates,
                                     float *mean_delta, float *variance_delta, int act, dnb_stream stream) {
    const char *what = "syncbn_backward_apply";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (total_count < 1) return fail(DNB_ERR_INVALID, "%s: total_count must be positive", what);
    if (filters == 0) return DNB_OK;
    if (!x || !delta || !dx || !reduced || !scales || !biases || !mean || !variance || !bias_updates ||
        !scale_updates || !mean_delta || !variance_delta)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x) && aligned16(delta) && (!y || aligned16(y)));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    return generic_bwd_apply(g, x, y, delta, dx, (float)total_count, reinterpret_cast<const double2 *>(reduced),
                             scales, biases, mean, variance, bias_updates, scale_updates, mean_delta, variance_delta,
                             act, sc, s);
}

}  // extern "C"
