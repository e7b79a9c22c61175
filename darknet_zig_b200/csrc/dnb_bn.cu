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
// written. The persistent kernel below (the sweep) keeps the second read off HBM: channels
// are taken in groups sized to a slice of the 126 MB L2; every CTA reduces its share of a
// group, the CTAs exchange tagged per-channel records through global memory, and each CTA
// then writes the outputs of its share, re-reading the inputs from L2 (see the comment
// above kSThreads). Every wait is bounded: a CTA that gives up sets the device error word and
// exits; the host reports DNB_ERR_TIMEOUT.
//
// Shapes the persistent kernel does not take (spatial % 4 != 0, unaligned pointers, more
// than 16 channel groups) run the generic three-launch path below, which also implements
// the split sync-BN entry points: per-channel partials -> (caller's collective) ->
// finalize + apply.
//
// Per-element arithmetic follows the reference CPU code (blas.zig:137-204) operation by
// operation without fused roundings (--fmad=false), so given the same per-channel
// statistics the outputs are bit-identical to it.
#include <math.h>

#include <algorithm>
#include <atomic>

#include "dnb_bn.cuh"

namespace dnb {
namespace {

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

// Forward finalize from a producer's statistics: npieces blocks [piece][filters] of (count, mean,
// M2). A block takes 32 channels and 32 slices of the pieces: lane l of warp w reads channel
// c0 + l of pieces w, w + 32, ... (a warp's loads are 32 consecutive channels of one piece) and
// keeps, in fp64 about a shift K (the channel's first piece's mean), n, sum n d and sum (M2 + n d^2)
// with d = mean_p - K; the 32 slices of a channel are then added in slice order through shared
// memory, and M2 = sum (M2 + n d^2) - (sum n d)^2 / n. One pass over the pieces, no division per
// piece, the same result on every launch.
constexpr int kPieceCh = 32, kPieceSlices = 32;
__global__ void __launch_bounds__(kPieceCh * kPieceSlices)
    k_fwd_finalize_pieces(int64_t filters, int64_t npieces, const double *pieces, const float *scales,
                          const float *biases, float *mean, float *var, float *rmean, float *rvar, float4 *tab) {
    __shared__ double3 part[kPieceSlices][kPieceCh];
    const int lane = threadIdx.x & 31, slice = threadIdx.x >> 5;
    const int64_t c = (int64_t)blockIdx.x * kPieceCh + lane;
    double sn = 0.0, snd = 0.0, sq = 0.0;
    // the shift: the first piece's mean when that piece is not empty (its mean is then data)
    const double K = c < filters && pieces[c * 3] > 0.0 ? pieces[c * 3 + 1] : 0.0;
    if (c < filters) {
#pragma unroll 4
        for (int64_t p = slice; p < npieces; p += kPieceSlices) {
            const double *q = pieces + (p * filters + c) * 3;
            const double nb = q[0], d = q[1] - K, m2 = q[2];
            if (nb > 0.0) {
                sn += nb;
                snd += nb * d;
                sq += m2 + nb * d * d;
            }
        }
    }
    part[slice][lane] = make_double3(sn, snd, sq);
    __syncthreads();
    if (slice != 0 || c >= filters) return;
    double n = 0.0, s1 = 0.0, s2 = 0.0;
    for (int w = 0; w < kPieceSlices; ++w) {
        const double3 t = part[w][lane];
        n += t.x;
        s1 += t.y;
        s2 += t.z;
    }
    double m2 = s2 - s1 * (s1 / n);
    if (m2 < 0.0) m2 = 0.0;
    const FwdClose f = fwd_close(K + s1 / n, m2, n);
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
    ConstDiv cdiv;  // division by the element count (normalize_delta)
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
    // dx = (g*gamma)*inv2 + vd*2*(x-m)/denom + md/denom (blas.zig:200), the division by cdiv
    __device__ static float num(float xv, const P &p) { return p.vd * 2.0f * (xv - p.m); }
    __device__ static float dx1(float gv, const P &p, float q) { return (gv * p.g) * p.inv2 + q + p.mdd; }
    __device__ float grad(float dv, float xv, float yv, const P &p) const {
        return bn_grad1<A, HASY>(dv, xv, yv, p, act);
    }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        const float4 q =
            div4_const(make_float4(num(v.x.x, p0), num(v.x.y, p1), num(v.x.z, p2), num(v.x.w, p3)), cdiv);
        st4(dx + 4 * i, make_float4(dx1(grad(v.d.x, v.x.x, v.y.x, p0), p0, q.x),
                                    dx1(grad(v.d.y, v.x.y, v.y.y, p1), p1, q.y),
                                    dx1(grad(v.d.z, v.x.z, v.y.z, p2), p2, q.z),
                                    dx1(grad(v.d.w, v.x.w, v.y.w, p3), p3, q.w)));
    }
    __device__ void scalar(int64_t i, P p) const {
        const float xv = x[i];
        dx[i] = dx1(grad(d[i], xv, HASY ? y[i] : 0.0f, p), p, div_const(num(xv, p), cdiv));
    }
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
    const ConstDiv cd = const_div(denom);
    return dispatch_act(act, [&]<int A>() {
        if (y)
            return chan::launch_chan(g.batch, g.filters, g.spatial,
                                     OpBwdApply<A, true>{x, y, delta, dx, tab, cd, act, al}, s, "bn backward apply");
        return chan::launch_chan(g.batch, g.filters, g.spatial,
                                 OpBwdApply<A, false>{x, y, delta, dx, tab, cd, act, al}, s, "bn backward apply");
    });
}

// ======================================================================================
// persistent fused kernel: the sweep
// ======================================================================================

// Everything the persistent kernel needs, by value. Partition arithmetic is 32-bit with
// FastDiv: the plan guarantees T * max(Ps, Pa) < 2^32.
struct PArgs {
    int64_t C, S;
    int N, K, U, NK;          // batch, pieces per plane, unit floats (S/K), units per channel
    int cg, G;                // channels per group, groups
    int Ps, depth;            // CTAs, lag (groups whose statistics run ahead of the outputs)
    int cap_units;            // most units a CTA's share of one group holds
    uint32_t T_full, T_last;  // units in a group (every group but the last / the last)
    FastDiv f_nk, f_k, f_ps, f_tfull, f_tlast;
    float denom;              // batch*spatial as f32 (normalize_delta's denominator)
    ConstDiv cdiv;            // division by denom, per element
    // tensors: fwd uses t0 = x; bwd uses t0 = delta, t1 = x, t2 = y (optional)
    const float *t0, *t1, *t2;
    float *out, *xnorm;
    const float *scales, *biases;
    float *mean, *var, *rmean, *rvar;
    const float *mean_in, *var_in;
    float *bias_upd, *scale_upd, *mean_delta, *var_delta;
    int act;
    unsigned long long *rec;  // this GPU's records [G][Ps][2 segments][4 words] (tagged words)
    size_t rec_words;         // words of the whole record area (cleared when the epoch wraps)
    int cpu, cpu_s;           // chunks per unit of the output pass / of the statistics pass
    FastDiv f_cpu, f_cpu_s;
    FastDiv f_u4;             // U / 4: float4s of a unit (the flat chunk cut)
    int nread, nwrite;        // streaming warps taking statistics / writing outputs (both kSWarps
                              // unless the roles are split: nread + nwrite = kSWarps)
    unsigned *sync;           // [0] launch epoch, [1] CTAs that have finished this launch
    unsigned *err, *abort_flag;
    unsigned long long wait_ns;
    // sync-BN across GPUs (xon, any world >= 1): every CTA stores its records of group g into
    // every rank's buffer (xrec[r]: a peer mapping, or this GPU's own buffer for r == rank),
    // tagged with the communicator's call number xtag; a rank reads them from its own buffer
    int xon, world, rank;
    int xpar;                 // call number & 1: which half of the buffers this launch uses
    int xpmax;                // CTAs a group's records have room for
    unsigned xtag;
    unsigned long long *xrec[kMaxRanks];
};

struct PPlan {
    bool ok = false;
    int K, U, cg, G, P, depth, cap_units, ctas_per_sm;
    size_t smem;
};


bool persistent_disabled() {
    const char *e = getenv("DNB_BN_PERSISTENT");
    return e && e[0] == '0';
}

// DNB_BN_SWEEP=0 turns the L2 sweep off (the staged kernel then takes its shapes).
bool sweep_disabled() {
    const char *e = getenv("DNB_BN_SWEEP");
    return e && e[0] == '0';
}
// DNB_BN_FLAT=0 keeps the sweep backward's per-unit chunk cut for every plane size.
bool flat_cut_disabled() {
    const char *e = getenv("DNB_BN_FLAT");
    return e && e[0] == '0';
}

// Every CTA owns the same balanced share of each channel group in both passes, and its
// warps are split by role. The 14 streaming warps reduce the groups (HBM reads) and write
// the outputs of each group once its parameters are known (the share re-read from L2),
// running `lag` groups of statistics ahead of the outputs; each warp walks its own chunks
// and meets the others only through shared-memory counters, so one warp's phase change
// never drains the whole CTA. The publisher warp takes a group's per-warp partials once
// every streaming warp has counted itself and stores the CTA's records (with a
// communicator: into every rank's buffer over NVLink), every word tagged with this launch's
// tag; the merger warp polls the records of its share's channels until all carry the tag,
// merges them and hands the apply parameters back through shared memory. No fence, counter
// or flag sits between a record's store and its merge, so a group's exchange costs one
// store and one poll round trip; it stays off the streaming path. Statistics loads carry
// an L2 evict_last policy, output-pass loads and stores evict_first, so a group stays in L2
// between its two passes. Every wait is bounded; on timeout the merger sets the device
// error word and tells the other warps to stop.

constexpr int kSThreads = 512;              // threads of a sweep CTA
constexpr int kSMinBlocks = 2;              // CTAs per SM the register budget is set for
constexpr int kSWarps = kSThreads / 32 - 2;  // streaming warps; then the publisher and the merger
constexpr unsigned kWaitSliceNs = 2000;      // longest suspension of one mbarrier try_wait
constexpr int kSplitReaders = 7;             // statistics warps when the roles are split

template <bool BWD, int A, bool HASY>
struct SweepKernel {
    // float4s per tensor in flight per thread: statistics loads come from HBM and get the
    // deeper unroll; output-pass loads hit L2
    static constexpr int UNROLL_S = BWD ? (HASY ? 2 : 2) : 4;
    static constexpr int UNROLL = BWD ? 2 : 4;
    static constexpr int CHUNK_S = 32 * UNROLL_S;  // float4s of one unit a statistics chunk holds
    static constexpr int CHUNK = 32 * UNROLL;      // the same for an output-pass chunk
    static constexpr int kRecWords = BWD ? 2 : 3;  // data words of a record

    // Per-group state, one buffer per group (G <= kMaxSweepGroups).
    struct Smem {
        uint32_t *utab;  // [G][cap_units] element offset of each unit of the share (< 2^32)
        float4 *wrec;    // [G][2 segments][kSWarps] per-warp partials
        float *ptab;     // [G][2 segments][8] apply parameters
        float4 *stab;    // [G][2 segments] forward parameters for the backward's stats
        float4 *ctab;    // [G][2 segments] channel inputs: (gamma, beta) or (mean, var, gamma, beta)
        double2 *lrec;   // [G][2 segments] this rank's merged records: (mean, M2) or (sum g, sum g(x-m))
        double *lcnt;    // [G][2 segments] elements behind the forward's records
        uint64_t *dbar;  // [G] mbarrier: every streaming warp has left its partials of group g
        uint64_t *rbar;  // [G] mbarrier: the parameters of group g are in ptab
        uint64_t *abar;  // [G] mbarrier (split roles): every output warp is done with group g
        int *stop;       // set by the merger warp when a wait gave up
    };
    __host__ __device__ static size_t smem_bytes(int cap_units, int groups) {
        return (((size_t)groups * cap_units * sizeof(uint32_t) + 15) & ~(size_t)15) +
               (size_t)groups * (2 * kSWarps * sizeof(float4) + 2 * sizeof(double2) + 2 * sizeof(double) +
                                 16 * sizeof(float) + 4 * sizeof(float4) + 3 * sizeof(uint64_t)) +
               16;
    }
    __device__ static Smem carve(const PArgs &a, unsigned char *raw) {
        const int G = a.G;
        Smem s;
        size_t o = 0;
        s.utab = reinterpret_cast<uint32_t *>(raw);
        o += ((size_t)G * a.cap_units * sizeof(uint32_t) + 15) & ~(size_t)15;
        s.wrec = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)G * 2 * kSWarps * sizeof(float4);
        s.lrec = reinterpret_cast<double2 *>(raw + o);
        o += (size_t)G * 2 * sizeof(double2);
        s.lcnt = reinterpret_cast<double *>(raw + o);
        o += (size_t)G * 2 * sizeof(double);
        s.stab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)G * 2 * sizeof(float4);
        s.ctab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)G * 2 * sizeof(float4);
        s.ptab = reinterpret_cast<float *>(raw + o);
        o += (size_t)G * 16 * sizeof(float);
        s.dbar = reinterpret_cast<uint64_t *>(raw + o);  // 16-byte aligned: every block above is
        o += (size_t)G * sizeof(uint64_t);
        s.rbar = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)G * sizeof(uint64_t);
        s.abar = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)G * sizeof(uint64_t);
        s.stop = reinterpret_cast<int *>(raw + o);
        return s;
    }

    // Bounded wait of a whole warp for the (only) phase of a per-group mbarrier; false if
    // the merger warp stopped the CTA or the wait gave up (the latter sets the device error
    // word). The waiting warp is suspended in try_wait (up to kWaitSliceNs at a time) rather
    // than spinning, so it takes no issue slots from the streaming warps.
    __device__ static bool wait_bar(const PArgs &a, const Smem &s, uint64_t *bar) {
        if (mbar_try_wait_ns(bar, 0u, 0u)) return true;
        const volatile int *stop = s.stop;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        while (!mbar_try_wait_ns(bar, 0u, kWaitSliceNs)) {
            if (*stop) return false;
            if (global_ns() > deadline) {
                if ((threadIdx.x & 31) == 0) {
                    atomicOr(a.err, DEVERR_WAIT_BARRIER);
                    atomicExch(a.abort_flag, 1u);
                }
                return false;
            }
        }
        return true;
    }

    // every thread: element offsets of the units of CTA rid's share of group g into table b
    __device__ static void tabulate(const PArgs &a, const Smem &s, int g, int rid, int b) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int n_units = (int)(sh.t1 - sh.t0);
        for (int u = threadIdx.x; u < n_units; u += kSThreads) {
            uint32_t cl, rem, n, k;
            a.f_nk.divmod(sh.t0 + u, cl, rem);
            a.f_k.divmod(rem, n, k);
            s.utab[b * a.cap_units + u] = (uint32_t)(((int64_t)n * a.C + sh.c0 + cl) * a.S + (int64_t)k * a.U);
        }
    }

    // threads t0, t0 + nt, ...: the per-channel inputs of the (at most two) channels of each
    // group's share, one (group, segment) per thread so that all loads are in flight at once;
    // the merger's closing then needs no global load between a group's records and its apply
    // parameters
    __device__ static void load_channels(const PArgs &a, const Smem &s, int rid, int t0, int nt) {
        for (int i = t0; i < 2 * a.G; i += nt) {
            const int g = i >> 1, j = i & 1;
            const Share sh = share_of(a, g, rid, a.f_ps);
            if (j >= sh.nseg) continue;
            const int64_t c = (int64_t)sh.c0 + sh.cfirst + j;
            if (BWD) {
                const float m = a.mean_in[c], v = a.var_in[c], gm = a.scales[c], bt = a.biases[c];
                s.ctab[i] = make_float4(m, v, gm, bt);
                // the forward's normalisation (batchnorm.zig:142), to recompute y from x
                s.stab[i] = make_float4(m, 1.0f / (sqrtf(v) + 0.000001f), gm, bt);
            } else {
                s.ctab[i] = make_float4(a.scales[c], a.biases[c], 0.0f, 0.0f);
            }
        }
    }

    // The share is cut into chunks of CH float4s; streaming warp w takes chunks w,
    // w + kSWarps, ... and lane l of a chunk holds its float4s l + 32 j, j < CH / 32. A
    // warp's chunks run through the share in order and no chunk spans two channels, so a
    // warp's segment changes at most once. Two cuts:
    //  * per unit: a unit is `cpu` chunks, the last one partial unless u4 (the float4s of a
    //    unit) is a multiple of CH;
    //  * flat (the backward, when u4 is not a multiple of CH): each segment's units are one
    //    run of float4s, cut into chunks regardless of unit ends, so no lane idles at the
    //    end of a unit (at 28x28 planes a per-unit cut leaves 60 of every 256 lanes idle).
    //    A lane then finds its unit with one FastDiv per float4.
    struct Walk {
        uint32_t n_chunks, nc0;  // chunks of the share, of its first segment
        uint32_t n0;             // units of the first segment
        uint32_t F0, F1;         // flat: float4s of the first / second segment
    };
    template <int CH, bool FLAT>
    __device__ static Walk walk_of(const PArgs &a, const Share &sh, int cpu) {
        Walk w;
        const uint32_t n = sh.nseg ? sh.t1 - sh.t0 : 0;
        w.n0 = sh.nseg == 2 ? sh.bnd - sh.t0 : n;
        if constexpr (!FLAT) {
            w.n_chunks = n * (uint32_t)cpu;
            w.nc0 = w.n0 * (uint32_t)cpu;
            w.F0 = w.F1 = 0;
            return w;
        }
        const uint32_t u4 = (uint32_t)a.U >> 2;
        w.F0 = w.n0 * u4;
        w.F1 = (n - w.n0) * u4;
        w.nc0 = (w.F0 + CH - 1) / CH;
        w.n_chunks = w.nc0 + (w.F1 + CH - 1) / CH;
        return w;
    }
    // element offsets of lane's float4s of chunk c (ok[j]: the float4 exists); returns the
    // chunk's segment
    template <int CH, bool FLAT>
    __device__ static int lanes_at(const PArgs &a, const Walk &w, const uint32_t *ut, const FastDiv &fcpu, uint32_t c,
                                   int lane, uint32_t (&off)[CH / 32], bool (&ok)[CH / 32]) {
        const uint32_t u4 = (uint32_t)a.U >> 2;
        if constexpr (!FLAT) {
            uint32_t uo, part;
            fcpu.divmod(c, uo, part);
            const uint32_t k = part * CH + lane;
            const uint32_t o = ut[uo] + 4 * k;
#pragma unroll
            for (int j = 0; j < CH / 32; ++j) {
                off[j] = o + 128 * j;
                ok[j] = k + 32 * j < u4;
            }
            return uo >= w.n0 ? 1 : 0;
        } else {
        const int seg = c >= w.nc0 ? 1 : 0;
        const uint32_t f0 = (seg ? c - w.nc0 : c) * CH + lane;
        const uint32_t F = seg ? w.F1 : w.F0, ub = seg ? w.n0 : 0;
#pragma unroll
        for (int j = 0; j < CH / 32; ++j) {
            const uint32_t f = f0 + 32 * j;
            uint32_t q, r;
            a.f_u4.divmod(f, q, r);
            ok[j] = f < F;
            off[j] = ok[j] ? ut[ub + q] + 4 * r : 0;
        }
        return seg;
        }
    }

    // streaming warps: statistics of CTA rid's share of group g (table b); each warp leaves
    // one partial per segment in s.wrec[b]
    template <bool FLAT>
    __device__ static void stats(const PArgs &a, const Smem &s, int g, int rid, int b) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
        const Walk w = walk_of<CHUNK_S, FLAT>(a, sh, a.cpu_s);
        const uint32_t n_chunks = w.n_chunks;
        const uint32_t *ut = s.utab + b * a.cap_units;
        const uint64_t pol = l2_evict_last();
        float4 rec[2];
        int seg = 0;
        uint32_t off[UNROLL_S];
        bool ok[UNROLL_S];
        if constexpr (!BWD) {
            Moments mo;
            float4 first = make_float4(0.0f, 0.0f, 0.0f, 0.0f);  // segment 0 once the warp moved on
            for (uint32_t c = warp; c < n_chunks; c += (uint32_t)a.nread) {
                const int cs = lanes_at<CHUNK_S, FLAT>(a, w, ut, a.f_cpu_s, c, lane, off, ok);
                if (cs != seg) {  // warp-uniform
                    first = mo.warp_summary();
                    mo = Moments();
                    seg = cs;
                }
                float4 v[UNROLL_S];
#pragma unroll
                for (int j = 0; j < UNROLL_S; ++j)
                    if (ok[j]) v[j] = ld4_hint(a.t0 + off[j], pol);
#pragma unroll
                for (int j = 0; j < UNROLL_S; ++j)
                    if (ok[j]) mo.add4(v[j]);
            }
            const float4 last = mo.warp_summary();
            rec[0] = seg ? first : last;
            rec[1] = seg ? last : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        } else {
            float s1 = 0.0f, s2 = 0.0f, f1 = 0.0f, f2 = 0.0f;  // f: segment 0 once the warp moved on
            for (uint32_t c = warp; c < n_chunks; c += (uint32_t)a.nread) {
                const int cs = lanes_at<CHUNK_S, FLAT>(a, w, ut, a.f_cpu_s, c, lane, off, ok);
                if (cs != seg) {
                    f1 = s1;
                    f2 = s2;
                    s1 = s2 = 0.0f;
                    seg = cs;
                }
                const float4 fp = s.stab[2 * b + seg];  // warp-uniform broadcast
                BwdParam p;
                p.m = fp.x;
                p.inv = fp.y;
                p.g = fp.z;
                p.b = fp.w;
                float4 d[UNROLL_S], xv[UNROLL_S], yv[UNROLL_S];
#pragma unroll
                for (int j = 0; j < UNROLL_S; ++j)
                    if (ok[j]) {
                        d[j] = ld4_hint(a.t0 + off[j], pol);
                        xv[j] = ld4_hint(a.t1 + off[j], pol);
                        if (HASY) yv[j] = ld4_hint(a.t2 + off[j], pol);
                    }
#pragma unroll
                for (int j = 0; j < UNROLL_S; ++j)
                    if (ok[j]) {
                        const float4 yy = HASY ? yv[j] : xv[j];
                        const float g0 = bn_grad1<A, HASY>(d[j].x, xv[j].x, yy.x, p, a.act);
                        const float g1 = bn_grad1<A, HASY>(d[j].y, xv[j].y, yy.y, p, a.act);
                        const float g2 = bn_grad1<A, HASY>(d[j].z, xv[j].z, yy.z, p, a.act);
                        const float g3 = bn_grad1<A, HASY>(d[j].w, xv[j].w, yy.w, p, a.act);
                        s1 += (g0 + g1) + (g2 + g3);
                        s2 += (g0 * (xv[j].x - p.m) + g1 * (xv[j].y - p.m)) +
                              (g2 * (xv[j].z - p.m) + g3 * (xv[j].w - p.m));
                    }
            }
            const float t1 = warp_sum(s1), t2 = warp_sum(s2);
            const float u1 = warp_sum(f1), u2 = warp_sum(f2);
            rec[0] = seg ? make_float4(u1, u2, 0.0f, 0.0f) : make_float4(t1, t2, 0.0f, 0.0f);
            rec[1] = seg ? make_float4(t1, t2, 0.0f, 0.0f) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        }
        if (lane == 0) {
            s.wrec[(2 * b + 0) * kSWarps + warp] = rec[0];
            s.wrec[(2 * b + 1) * kSWarps + warp] = rec[1];
            __threadfence_block();
            mbar_arrive(&s.dbar[b]);  // releases the partials above
        }
        __syncwarp();
    }

    // publisher warp: one record per segment from the streaming warps' partials of group g
    // (buffer b), written to a.rec; lane 0 then publishes them and counts the CTA
    __device__ static void publish(const PArgs &a, const Smem &s, int g, int rid, int b, unsigned tag) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int lane = threadIdx.x & 31;
        for (int j = 0; j < sh.nseg; ++j) {
            float4 q = lane < a.nread ? s.wrec[(2 * b + j) * kSWarps + lane] : make_float4(0, 0, 0, 0);
            if constexpr (!BWD) {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const float cb = __shfl_xor_sync(0xffffffffu, q.x, o);
                    const float mb = __shfl_xor_sync(0xffffffffu, q.y, o);
                    const float qb = __shfl_xor_sync(0xffffffffu, q.z, o);
                    chan_merge(q.x, q.y, q.z, cb, mb, qb);
                }
            } else {
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    q.x += __shfl_xor_sync(0xffffffffu, q.x, o);
                    q.y += __shfl_xor_sync(0xffffffffu, q.y, o);
                }
            }
            if (a.xon) {
                // the butterfly leaves lanes with values that differ in the last bits (Chan's
                // merge is not symmetric): every rank must get lane 0's record
                q.x = __shfl_sync(0xffffffffu, q.x, 0);
                q.y = __shfl_sync(0xffffffffu, q.y, 0);
                q.z = __shfl_sync(0xffffffffu, q.z, 0);
                q.w = __shfl_sync(0xffffffffu, q.w, 0);
                // lane r stores the record into rank r's buffer
                if (lane < a.world) st_record<kRecWords>(a.xrec[lane] + xslot(a, g, a.rank, rid, j), q, tag, true);
            } else if (lane == 0) {
                st_record<kRecWords>(a.rec + (((size_t)g * a.Ps + rid) * 2 + j) * 4, q, tag, false);
            }
        }
        __syncwarp();
    }

    // first word of the record (group g, segment j) of CTA p of rank r in an exchange buffer
    __device__ static size_t xslot(const PArgs &a, int g, int r, int p, int j) {
        return (((((size_t)a.xpar * kMaxSweepGroups + g) * a.world + r) * a.xpmax + p) * 2 + j) * 4;
    }

    // merger warp: merge the records of the (at most two) channels of CTA rid's share of
    // group g into s.lrec[g] -- this GPU's CTAs' records, or with a communicator every
    // rank's, in the same order on every rank (so every rank gets the same statistics).
    // Records of CTAs between the channel's first and last owner that hold no unit of it (a
    // group with fewer units than CTAs) are skipped. The lanes poll their records until all
    // carry this launch's tag (bounded; false when the wait gave up or the launch aborted).
    __device__ static bool merge_local(const PArgs &a, const Smem &s, int g, int rid, unsigned tag) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int lane = threadIdx.x & 31;
        for (int j = 0; j < sh.nseg; ++j) {
            const int cl = sh.cfirst + j;
            const uint32_t ua = (uint32_t)cl * a.NK, ub = ua + a.NK;
            const int plo = owner_of(a, g, ua, a.Ps), phi = owner_of(a, g, ub - 1, a.Ps);
            const int per_rank = phi - plo + 1;
            const int nrec = a.xon ? per_rank * a.world : per_rank;
            // 1: the record is loaded and complete; 0: no record to merge; -1: not yet written
            auto load = [&](int idx, float4 &dst) -> int {
                int q = 0, k = idx;
                if (a.xon) {
                    q = idx / per_rank;
                    k = idx - q * per_rank;
                }
                const int p = plo + k;
                const Share o = share_of(a, g, p, a.f_ps);
                const uint32_t lo = ua > o.t0 ? ua : o.t0, hi = ub < o.t1 ? ub : o.t1;
                if (hi <= lo) return 0;
                const int oj = cl - o.cfirst;
                const bool done =
                    a.xon ? ld_record<kRecWords>(a.xrec[a.rank] + xslot(a, g, q, p, oj), tag, true, dst)
                          : ld_record<kRecWords>(a.rec + (((size_t)g * a.Ps + p) * 2 + oj) * 4, tag, false, dst);
                return done ? 1 : -1;
            };
            constexpr int R = 2;  // records held per lane: one L2 round trip up to 64 records
            float4 r[R];
            bool have[R];
            {
                const unsigned long long deadline = global_ns() + a.wait_ns;
                unsigned polls = 0;
                for (;;) {
                    bool complete = true;
#pragma unroll
                    for (int k = 0; k < R; ++k) {
                        const int idx = lane + 32 * k;
                        const int st = idx < nrec ? load(idx, r[k]) : 0;
                        have[k] = st == 1;
                        complete = complete && st >= 0;
                    }
                    for (int idx = lane + 32 * R; idx < nrec; idx += 32) {
                        float4 t;
                        complete = complete && load(idx, t) >= 0;
                    }
                    if (__all_sync(0xffffffffu, complete)) break;
                    int give_up = 0;
                    if (lane == 0) {
                        // the abort word is a second round trip: read it on every 8th poll
                        if ((++polls & 7u) == 0 && ld_volatile(a.abort_flag)) give_up = 1;
                        if (global_ns() > deadline) {
                            atomicOr(a.err, a.xon ? DEVERR_WAIT_PEER : DEVERR_WAIT_BARRIER);
                            atomicExch(a.abort_flag, 1u);
                            give_up = 1;
                        }
                    }
                    if (__shfl_sync(0xffffffffu, give_up, 0)) return false;
                    __nanosleep(20);
                }
            }
            double2 mine;
            if constexpr (!BWD) {
                double sn = 0.0, smn = 0.0;
#pragma unroll
                for (int k = 0; k < R; ++k)
                    if (have[k]) {
                        sn += (double)r[k].x;
                        smn += (double)r[k].x * (double)r[k].y;
                    }
                for (int idx = lane + 32 * R; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    sn += (double)t.x;
                    smn += (double)t.x * (double)t.y;
                }
                sn = warp_sum(sn);
                const double mu = warp_sum(smn) / sn;
                double m2 = 0.0;
#pragma unroll
                for (int k = 0; k < R; ++k)
                    if (have[k]) {
                        const double d = (double)r[k].y - mu;
                        m2 += (double)r[k].z + (double)r[k].x * d * d;
                    }
                for (int idx = lane + 32 * R; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    const double d = (double)t.y - mu;
                    m2 += (double)t.z + (double)t.x * d * d;
                }
                m2 = warp_sum(m2);
                mine = make_double2(mu, m2);
                if (lane == 0) s.lcnt[2 * g + j] = sn;
            } else {
                double s1 = 0.0, s2 = 0.0;
#pragma unroll
                for (int k = 0; k < R; ++k)
                    if (have[k]) {
                        s1 += (double)r[k].x;
                        s2 += (double)r[k].y;
                    }
                for (int idx = lane + 32 * R; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    s1 += (double)t.x;
                    s2 += (double)t.y;
                }
                mine = make_double2(warp_sum(s1), warp_sum(s2));
            }
            if (lane == 0) s.lrec[2 * g + j] = mine;
        }
        __syncwarp();
        return true;
    }

    // merger warp: the merged statistics of the channels of CTA rid's share of group g
    // closed into the apply parameters s.ptab[g]; the CTA owning a channel's first unit
    // writes the per-channel outputs.
    // (lane 0; from shared memory only) the apply parameters of group g into s.ptab[g]
    __device__ static void finalize(const PArgs &a, const Smem &s, int g, int rid) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int lane = threadIdx.x & 31;
        if (lane == 0)
            for (int j = 0; j < sh.nseg; ++j) {
                const double2 tot = s.lrec[2 * g + j];
                const float4 ci = s.ctab[2 * g + j];
                float *out = s.ptab + (2 * g + j) * 8;
                if constexpr (!BWD) {
                    const FwdClose f = fwd_close(tot.x, tot.y, s.lcnt[2 * g + j]);
                    *reinterpret_cast<float4 *>(out) = make_float4(f.m, f.inv, ci.x, ci.y);
                } else {
                    *reinterpret_cast<BwdParam *>(out) = bwd_params(tot.x, tot.y, ci.x, ci.y, ci.z, ci.w, a.denom);
                }
            }
        __syncwarp();
    }

    // (lane 0, after the parameters are out) the per-channel outputs of group g, written by
    // the CTA owning the channel's first unit
    __device__ static void write_channels(const PArgs &a, const Smem &s, int g, int rid) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int lane = threadIdx.x & 31;
        if (lane == 0)
            for (int j = 0; j < sh.nseg; ++j) {
                const int cl = sh.cfirst + j;
                const int64_t c = (int64_t)sh.c0 + cl;
                if (owner_of(a, g, (uint32_t)cl * a.NK, a.Ps) != rid) continue;
                const double2 tot = s.lrec[2 * g + j];
                if constexpr (!BWD) {
                    const FwdClose f = fwd_close(tot.x, tot.y, s.lcnt[2 * g + j]);
                    const float rm = a.rmean[c], rv = a.rvar[c];
                    a.mean[c] = f.m;
                    a.var[c] = f.var;
                    a.rmean[c] = rolling(rm, f.m);
                    a.rvar[c] = rolling(rv, f.var);
                } else {
                    const float4 ci = s.ctab[2 * g + j];
                    float md;
                    const BwdParam p = bwd_params(tot.x, tot.y, ci.x, ci.y, ci.z, ci.w, a.denom, &md);
                    bwd_write(tot.x, tot.y, p, md, a.bias_upd, a.scale_upd, a.mean_delta, a.var_delta, c);
                }
            }
        __syncwarp();
    }

    // streaming warps: outputs of CTA rid's share of group g (table b, parameters s.ptab[b])
    template <bool FLAT>
    __device__ static void apply(const PArgs &a, const Smem &s, int g, int rid, int b) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        if (sh.nseg == 0) return;
        const int warp = (threadIdx.x >> 5) - (a.nwrite < kSWarps ? a.nread : 0), lane = threadIdx.x & 31;
        const Walk w = walk_of<CHUNK, FLAT>(a, sh, a.cpu);
        const uint32_t n_chunks = w.n_chunks;
        const uint32_t *ut = s.utab + b * a.cap_units;
        const float *ptab = s.ptab + 16 * b;
        const uint64_t pol = l2_evict_first();
        uint32_t offs[UNROLL];
        bool ok[UNROLL];
        if constexpr (!BWD) {
            for (uint32_t c = warp; c < n_chunks; c += (uint32_t)a.nwrite) {
                const int cs = lanes_at<CHUNK, FLAT>(a, w, ut, a.f_cpu, c, lane, offs, ok);
                const float4 p = *reinterpret_cast<const float4 *>(ptab + 8 * cs);
                float4 v[UNROLL];
#pragma unroll
                for (int j = 0; j < UNROLL; ++j)
                    if (ok[j]) v[j] = ld4_hint(a.t0 + offs[j], pol);
#pragma unroll
                for (int j = 0; j < UNROLL; ++j)
                    if (ok[j]) {
                        const uint32_t off = offs[j];
                        if (a.xnorm)
                            st4_hint(a.xnorm + off,
                                     make_float4((v[j].x - p.x) * p.y, (v[j].y - p.x) * p.y, (v[j].z - p.x) * p.y,
                                                 (v[j].w - p.x) * p.y),
                                     pol);
                        st4_hint(a.out + off,
                                 make_float4(bn_fwd1<A>(v[j].x, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v[j].y, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v[j].z, p.x, p.y, p.z, p.w, a.act),
                                             bn_fwd1<A>(v[j].w, p.x, p.y, p.z, p.w, a.act)),
                                 pol);
                    }
            }
        } else {
            for (uint32_t c = warp; c < n_chunks; c += (uint32_t)a.nwrite) {
                const int cs = lanes_at<CHUNK, FLAT>(a, w, ut, a.f_cpu, c, lane, offs, ok);
                const BwdParam p = *reinterpret_cast<const BwdParam *>(ptab + 8 * cs);
                float4 d[UNROLL], xv[UNROLL], yv[UNROLL];
#pragma unroll
                for (int j = 0; j < UNROLL; ++j)
                    if (ok[j]) {
                        d[j] = ld4_hint(a.t0 + offs[j], pol);
                        xv[j] = ld4_hint(a.t1 + offs[j], pol);
                        if (HASY) yv[j] = ld4_hint(a.t2 + offs[j], pol);
                    }
#pragma unroll
                for (int j = 0; j < UNROLL; ++j)
                    if (ok[j]) {
                        const float4 yy = HASY ? yv[j] : xv[j];
                        st4_hint(a.out + offs[j], bn_dx4_p(bn_grad4<A, HASY>(d[j], xv[j], yy, p, a.act), xv[j], p, a),
                                 pol);
                    }
            }
        }
    }
};

// The roles of a sweep CTA; each returns when its work is done or a wait gave up.
template <bool BWD, int A, bool HASY>
__device__ void sweep_publisher(const PArgs &a, const typename SweepKernel<BWD, A, HASY>::Smem &s, int rid,
                                unsigned tag) {
    using K = SweepKernel<BWD, A, HASY>;
    // groups in order, as soon as every streaming warp's partials are in
    for (int g = 0; g < a.G; ++g) {
        if (!K::wait_bar(a, s, &s.dbar[g])) return;
        K::publish(a, s, g, rid, g, tag);
    }
}
template <bool BWD, int A, bool HASY>
__device__ void sweep_merger(const PArgs &a, const typename SweepKernel<BWD, A, HASY>::Smem &s, int rid,
                             unsigned tag) {
    using K = SweepKernel<BWD, A, HASY>;
    const int lane = threadIdx.x & 31;
    if (!BWD) {
        K::load_channels(a, s, rid, lane, 32);
        __syncwarp();
    }
    // groups in order, once the records of the share's channels (of every rank) are in
    for (int g = 0; g < a.G; ++g) {
        if (!K::merge_local(a, s, g, rid, tag)) {
            if (lane == 0) *reinterpret_cast<volatile int *>(s.stop) = 1;
            return;
        }
        K::finalize(a, s, g, rid);  // ends with __syncwarp: the lanes' ptab writes are in
        if (lane == 0) mbar_arrive(&s.rbar[g]);
        __syncwarp();
        K::write_channels(a, s, g, rid);
    }
}
template <bool BWD, int A, bool HASY, bool FLAT>
__device__ void sweep_streamer(const PArgs &a, const typename SweepKernel<BWD, A, HASY>::Smem &s, int rid) {
    using K = SweepKernel<BWD, A, HASY>;
    // statistics of groups 0 .. lag-1, then per group g the statistics of group g + lag
    // followed by the outputs of group g
    if (a.nwrite < kSWarps) {
        // split roles: warps below nread read the statistics of every group, the others write
        // the outputs; a reader starts group h once the writers are done with group
        // h - lag - 1, so at most lag + 1 groups wait in L2
        const int warp = threadIdx.x >> 5;
        if (warp < a.nread) {
            for (int h = 0; h < a.G; ++h) {
                if (h > a.depth && !K::wait_bar(a, s, &s.abar[h - a.depth - 1])) return;
                K::template stats<FLAT>(a, s, h, rid, h);
            }
        } else {
            for (int g = 0; g < a.G; ++g) {
                if (!K::wait_bar(a, s, &s.rbar[g])) return;
                K::template apply<FLAT>(a, s, g, rid, g);
                __syncwarp();
                if ((threadIdx.x & 31) == 0) mbar_arrive(&s.abar[g]);
            }
        }
        return;
    }
    for (int h = 0; h < a.depth && h < a.G; ++h) K::template stats<FLAT>(a, s, h, rid, h);
    for (int g = 0; g < a.G; ++g) {
        if (g + a.depth < a.G) K::template stats<FLAT>(a, s, g + a.depth, rid, g + a.depth);
        if (!K::wait_bar(a, s, &s.rbar[g])) return;  // group g's parameters
        K::template apply<FLAT>(a, s, g, rid, g);
    }
}

template <bool BWD, int A, bool HASY, bool FLAT>
__global__ void __launch_bounds__(kSThreads, kSMinBlocks) k_bn_sweep(PArgs a) {
    using K = SweepKernel<BWD, A, HASY>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const typename K::Smem s = K::carve(a, smem_raw);
    __shared__ unsigned s_epoch;
    __shared__ int s_exited;
    const int rid = (int)blockIdx.x;
    if (threadIdx.x == 0) {
        s_epoch = ld_volatile(&a.sync[0]);
        *s.stop = 0;
        s_exited = 0;
    }
    if (threadIdx.x < a.G) {
        mbar_init(&s.dbar[threadIdx.x], (unsigned)a.nread);
        mbar_init(&s.abar[threadIdx.x], (unsigned)a.nwrite);
        mbar_init(&s.rbar[threadIdx.x], 1);
    }
    for (int g = 0; g < a.G; ++g) K::tabulate(a, s, g, rid, g);
    // the backward's statistics pass needs the forward's parameters at once; the forward's
    // channel inputs are only the merger's, which loads them itself off the prologue
    if (BWD) K::load_channels(a, s, rid, threadIdx.x, kSThreads);
    __syncthreads();
    // this launch's record tag: the communicator's call number, or the launch epoch + 1
    // (never 0, the tag of a cleared record)
    const unsigned epoch = s_epoch;
    const unsigned tag = a.xon ? a.xtag : epoch + 1u;
    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    // The epoch advances once per launch, after every CTA has read it; the next launch on
    // this stream starts after this one has ended. In the launch whose successor's tag would
    // wrap to 0 the record area is cleared first, once no CTA reads records any more: there
    // the last warp of the last CTA to finish does it (once per 2^32 - 1 launches). In every
    // other launch the last CTA whose publisher is done does it, off the kernel's tail.
    const bool wraps = epoch + 2u == 0u;
    if (warp == kSWarps) {
        sweep_publisher<BWD, A, HASY>(a, s, rid, tag);
        __syncwarp();
        if (!wraps && lane == 0 && atomicAdd(&a.sync[1], 1u) == (unsigned)a.Ps - 1u) {
            a.sync[1] = 0u;
            a.sync[0] = epoch + 1u;
        }
    } else if (warp == kSWarps + 1) {
        sweep_merger<BWD, A, HASY>(a, s, rid, tag);
    } else {
        sweep_streamer<BWD, A, HASY, FLAT>(a, s, rid);
    }
    if (!wraps) return;
    __syncwarp();
    int last = 0;
    if (lane == 0 && atomicAdd(&s_exited, 1) == kSThreads / 32 - 1)
        last = atomicAdd(&a.sync[1], 1u) == (unsigned)a.Ps - 1u;
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    for (size_t i = lane; i < a.rec_words; i += 32) a.rec[i] = 0ull;
    __syncwarp();
    if (lane == 0) {
        a.sync[1] = 0u;
        a.sync[0] = 0u;
    }
}

// Sweep plan: P = CTAs per SM x SMs; channel groups whose inputs fill about
// DNB_BN_GROUP_MB per input tensor (default 32 MiB forward, 16 MiB backward), at most
// kMaxSweepGroups of them; lag = groups whose statistics run ahead of the outputs, as many
// as keep lag + 1 groups within DNB_BN_L2_MB per input tensor (default 64 MiB forward,
// 32 MiB backward) of L2, so that the grid exchange of a group is hidden behind later
// statistics passes (or, when the whole input fits, every statistics pass runs before the
// first output pass). The defaults are the fastest measured at BASELINE configs 0/1 on the
// B200: the forward's single input fits L2 in two groups; the backward's two inputs do not,
// and smaller groups with a lag of one keep its output pass in L2; units of U = spatial/K floats with K the smallest divisor giving
// >= 8 units per CTA in a group (U >= 256 floats); cg <= P keeps a share within two
// channels.
template <bool BWD, bool HASY>
PPlan plan_sweep(int64_t batch, int64_t filters, int64_t spatial, const DeviceState *ds, int occupancy) {
    using K = SweepKernel<BWD, DNB_ACT_LEAKY, HASY>;
    constexpr int nt = BWD ? (HASY ? 3 : 2) : 1;
    PPlan pl;
    if (spatial % 4 != 0 || batch <= 0 || filters <= 0) return pl;
    int ctas = occupancy < 1 ? 1 : occupancy;
    if (ctas > 2048 / kSThreads) ctas = 2048 / kSThreads;
    const int64_t P = (int64_t)ds->sm_count * ctas;
    const int64_t bytes_per_channel = batch * spatial * 4 * nt;
    const int64_t budget = ((int64_t)env_int("DNB_BN_GROUP_MB", BWD ? 16 : 32, 1, 4096) << 20) * nt;
    int64_t cg = budget / bytes_per_channel;
    if (cg < 1) cg = 1;
    if (cg > P) cg = P;
    if (cg > filters) cg = filters;
    int64_t G = (filters + cg - 1) / cg;
    cg = (filters + G - 1) / G;
    G = (filters + cg - 1) / cg;
    if (G > kMaxSweepGroups) return pl;
    int64_t k = 0;
    for (int64_t kk = 1; kk <= spatial; ++kk) {
        if (spatial % kk || (spatial / kk) % 4) continue;
        if (k == 0) k = kk;
        if (spatial / kk < 256) break;
        k = kk;
        if (cg * batch * kk >= 8 * P) break;
    }
    if (k == 0) return pl;
    const int64_t U = spatial / k, NK = batch * k, T = cg * NK;
    if ((uint64_t)T * (uint64_t)P >= (1ull << 32) - (uint64_t)P) return pl;
    if ((uint64_t)batch * (uint64_t)filters * (uint64_t)spatial >= (1ull << 32)) return pl;  // 32-bit offsets
    const int64_t share = (T + P - 1) / P;
    pl.K = (int)k;
    pl.U = (int)U;
    pl.cg = (int)cg;
    pl.G = (int)G;
    pl.P = (int)P;
    const int64_t l2 = ((int64_t)env_int("DNB_BN_L2_MB", BWD ? 32 : 64, 1, 4096) << 20) * nt;
    int64_t lag = l2 / (cg * bytes_per_channel) - 1;
    if (lag > G - 1) lag = G - 1;
    if (lag < 0) lag = 0;
    pl.depth = (int)lag;
    pl.cap_units = (int)share;
    pl.ctas_per_sm = ctas;
    pl.smem = K::smem_bytes(pl.cap_units, pl.G);
    size_t per_cta = (size_t)ds->smem_per_sm / ctas - (size_t)ds->smem_reserved - 256;
    if (per_cta > (size_t)ds->max_smem_optin) per_cta = (size_t)ds->max_smem_optin;
    pl.ok = pl.smem <= per_cta;
    return pl;
}

// Fills the partition fields of `a` from a plan whose two roles have ps and pa CTAs.
void fill_partition(PArgs &a, const PPlan &pl, int64_t batch, int64_t filters, int64_t spatial) {
    a.C = filters;
    a.S = spatial;
    a.N = (int)batch;
    a.K = pl.K;
    a.U = pl.U;
    a.NK = (int)(batch * pl.K);
    a.cg = pl.cg;
    a.G = pl.G;
    a.Ps = pl.P;
    a.depth = pl.depth;
    a.cap_units = pl.cap_units;
    a.T_full = (uint32_t)pl.cg * (uint32_t)a.NK;
    a.T_last = (uint32_t)(filters - (int64_t)(pl.G - 1) * pl.cg) * (uint32_t)a.NK;
    a.f_nk = FastDiv((uint32_t)a.NK);
    a.f_k = FastDiv((uint32_t)pl.K);
    a.f_ps = FastDiv((uint32_t)pl.P);
    a.f_tfull = FastDiv(a.T_full);
    a.f_tlast = FastDiv(a.T_last);
    a.denom = (float)(spatial * batch);
    a.cdiv = const_div(a.denom);
}

template <bool BWD, bool HASY>
dnb_status run_sweep(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                     bool *launched, const char *what, const CommView *cv = nullptr) {
    *launched = false;
    if (sweep_disabled()) return DNB_OK;
    PArgs a{};
    a.t0 = io.t0;
    a.t1 = io.t1;
    a.t2 = io.t2;
    a.out = io.out;
    a.xnorm = io.xnorm;
    a.scales = io.scales;
    a.biases = io.biases;
    a.mean = io.mean;
    a.var = io.var;
    a.rmean = io.rmean;
    a.rvar = io.rvar;
    a.mean_in = io.mean_in;
    a.var_in = io.var_in;
    a.bias_upd = io.bias_upd;
    a.scale_upd = io.scale_upd;
    a.mean_delta = io.mean_delta;
    a.var_delta = io.var_delta;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    return dispatch_act(act, [&]<int A>() -> dnb_status {
        // The plan (its unit size) decides the chunk cut, and so the kernel; both
        // instantiations have the same launch bounds and static shared memory.
        constexpr int chunk = SweepKernel<BWD, A, HASY>::CHUNK;
        static_assert(chunk == SweepKernel<BWD, A, HASY>::CHUNK_S, "one chunk cut for both passes");
        // CTAs one SM holds with up to 16 KB of dynamic shared memory, per device and
        // kernel (a plan needs less unless its shares are thousands of units long; larger
        // plans are refused below, so the default dynamic shared-memory limit always
        // suffices and no per-device attribute is set). Cached as occupancy + 1; concurrent
        // first calls store the same value.
        static std::atomic<int> occ_by_device[kMaxDevices][2];
        auto occupancy_of = [&](auto kern, int flat) -> dnb_status {
            if (occ_by_device[ds->device][flat].load(std::memory_order_relaxed) == 0) {
                int o = 0;
                DNB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&o, kern, kSThreads, 16384));
                occ_by_device[ds->device][flat].store(o + 1, std::memory_order_relaxed);
            }
            return DNB_OK;
        };
        DNB_TRY(occupancy_of(k_bn_sweep<BWD, A, HASY, false>, 0));
        int occ1 = occ_by_device[ds->device][0].load(std::memory_order_relaxed);
        if constexpr (BWD) {
            DNB_TRY(occupancy_of(k_bn_sweep<BWD, A, HASY, true>, 1));
            occ1 = std::min(occ1, occ_by_device[ds->device][1].load(std::memory_order_relaxed));
        }
        const int occupancy = occ1 - 1;
        if (occupancy < 1) return DNB_OK;
        const PPlan pl = plan_sweep<BWD, HASY>(batch, filters, spatial, ds, occupancy);
        if (!pl.ok || pl.smem > 16384) return DNB_OK;
        Workspace *ws = nullptr;
        DNB_TRY(workspace(stream, 0, &ws, (size_t)pl.G * pl.P * 2 * 4));
        fill_partition(a, pl, batch, filters, spatial);
        a.cpu = (pl.U / 4 + chunk - 1) / chunk;
        a.f_cpu = FastDiv((uint32_t)a.cpu);
        a.cpu_s = a.cpu;
        a.f_cpu_s = a.f_cpu;
        // the flat cut pays in the backward only: measured on the B200 at [128,256,28,28]
        // the backward ran 110.2 us flat against 114.0 us per unit, the forward (whose
        // statistics pass streams at HBM speed with less arithmetic to hide the extra index
        // work behind) 65.1 us against 55.5 us
        [[maybe_unused]] const bool flat = BWD && (pl.U / 4) % chunk != 0 && !flat_cut_disabled();
        a.f_u4 = FastDiv((uint32_t)(pl.U / 4));
        // Split roles: kSplitReaders streaming warps take the statistics and the others write
        // the outputs, concurrently, so HBM reads go on while outputs are written from L2. It
        // pays in the backward over many groups: measured on the B200, [128,256,28,28] (7
        // groups) 90.8 against 95.5 us, [256,256,28,28] (13) 175.0 against 181.1 us, and
        // within 0.6 % either way at [128,196,32,32] and [128,64,56,56] (7); with 4 groups it
        // lost ([128,128,32,32] 55.7 against 52.5 us), and every forward measured slower.
        // DNB_BN_SPLIT=r forces r readers (0: every streaming warp does both passes).
        const int split_auto = BWD && pl.G >= 6 ? kSplitReaders : 0;
        a.nread = env_int("DNB_BN_SPLIT", split_auto, 0, kSWarps - 1);
        a.nwrite = a.nread ? kSWarps - a.nread : kSWarps;
        if (!a.nread) a.nread = kSWarps;
        a.act = act;
        a.rec = ws->recs;
        a.rec_words = ws->rec_words;
        a.sync = ws->sync;
        a.err = ds->error_word;
        a.abort_flag = ds->abort_flag;
        a.wait_ns = wait_limit_ns();
        a.xon = 0;
        a.world = 1;
        if (cv) {
            if (pl.P > cv->pmax || pl.G > kMaxSweepGroups)
                return fail(DNB_ERR_UNSUPPORTED, "%s: plan exceeds the communicator's buffers", what);
            a.xon = 1;
            a.world = cv->world;
            a.rank = cv->rank;
            a.xpar = (int)(cv->tag & 1u);
            a.xpmax = cv->pmax;
            a.xtag = cv->tag;
            for (int r = 0; r < cv->world; ++r) a.xrec[r] = cv->rec[r];
            // normalize_delta divides by the element count of the whole batch
            a.denom = (float)(batch * spatial * cv->world);
            a.cdiv = const_div(a.denom);
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)pl.P);
        cfg.blockDim = dim3(kSThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        if constexpr (BWD) {
            if (flat)
                DNB_CUDA(cudaLaunchKernelEx(&cfg, k_bn_sweep<BWD, A, HASY, true>, a));
            else
                DNB_CUDA(cudaLaunchKernelEx(&cfg, k_bn_sweep<BWD, A, HASY, false>, a));
        } else {
            DNB_CUDA(cudaLaunchKernelEx(&cfg, k_bn_sweep<BWD, A, HASY, false>, a));
        }
        *launched = true;
        return after_launch(stream, what);
    });
}

}  // namespace
}  // namespace dnb

using namespace dnb;

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
        BnIO a;
        a.t0 = x;
        a.out = y;
        a.xnorm = x_norm;
        a.scales = scales;
        a.biases = biases;
        a.mean = mean;
        a.var = variance;
        a.rmean = rolling_mean;
        a.rvar = rolling_variance;
        bool launched = false;
        if (!small_disabled()) DNB_TRY((run_small<false, false>(batch, filters, spatial, act, a, s, &launched, what)));
        if (launched) return DNB_OK;
        DNB_TRY((run_sweep<false, false>(batch, filters, spatial, act, a, s, &launched, what)));
        if (launched) return DNB_OK;
        if (!cluster_disabled())
            DNB_TRY((run_cluster<false, false>(batch, filters, spatial, act, a, s, &launched, what, nullptr)));
        if (launched) return DNB_OK;
        if (!stage_disabled()) DNB_TRY((run_stage<false, false>(batch, filters, spatial, act, a, s, &launched, what,
                                                                nullptr)));
        if (launched) return DNB_OK;
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
        BnIO a;
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
        bool launched = false;
        if (!small_disabled()) {
            if (y)
                DNB_TRY((run_small<true, true>(batch, filters, spatial, act, a, s, &launched, what)));
            else
                DNB_TRY((run_small<true, false>(batch, filters, spatial, act, a, s, &launched, what)));
            if (launched) return DNB_OK;
        }
        if (y)
            DNB_TRY((run_sweep<true, true>(batch, filters, spatial, act, a, s, &launched, what)));
        else
            DNB_TRY((run_sweep<true, false>(batch, filters, spatial, act, a, s, &launched, what)));
        if (launched) return DNB_OK;
        if (!cluster_disabled()) {
            if (y)
                DNB_TRY((run_cluster<true, true>(batch, filters, spatial, act, a, s, &launched, what, nullptr)));
            else
                DNB_TRY((run_cluster<true, false>(batch, filters, spatial, act, a, s, &launched, what, nullptr)));
            if (launched) return DNB_OK;
        }
        if (!launched && !stage_disabled()) {
            if (y)
                DNB_TRY((run_stage<true, true>(batch, filters, spatial, act, a, s, &launched, what, nullptr)));
            else
                DNB_TRY((run_stage<true, false>(batch, filters, spatial, act, a, s, &launched, what, nullptr)));
        }
        if (launched) return DNB_OK;
    }
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x) && aligned16(delta) && (!y || aligned16(y)));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    DNB_TRY(generic_bwd_partials(g, x, y, delta, mean, variance, scales, biases, act, sc, s));
    return generic_bwd_apply(g, x, y, delta, dx, (float)(spatial * batch), sc.local, scales, biases, mean, variance,
                             bias_updates, scale_updates, mean_delta, variance_delta, act, sc, s);
}

dnb_status dnb_syncbn_act_forward_train(dnb_comm comm, const float *x, float *y, float *x_norm, int64_t batch,
                                        int64_t filters, int64_t spatial, const float *scales, const float *biases,
                                        float *mean, float *variance, float *rolling_mean,
                                        float *rolling_variance, int act, dnb_stream stream) {
    const char *what = "syncbn_act_forward_train";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (filters == 0) return DNB_OK;
    if (!x || !y || !scales || !biases || !mean || !variance || !rolling_mean || !rolling_variance)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    CommView cv;
    DNB_TRY(comm_next(comm, &cv));
    if (filters > cv.cmax) return fail(DNB_ERR_UNSUPPORTED, "%s: %lld channels, communicator holds %lld", what,
                                       (long long)filters, (long long)cv.cmax);
    if (!(aligned16(x) && aligned16(y) && (!x_norm || aligned16(x_norm))))
        return fail(DNB_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned", what);
    BnIO a;
    a.t0 = x;
    a.out = y;
    a.xnorm = x_norm;
    a.scales = scales;
    a.biases = biases;
    a.mean = mean;
    a.var = variance;
    a.rmean = rolling_mean;
    a.rvar = rolling_variance;
    bool launched = false;
    DNB_TRY((run_sweep<false, false>(batch, filters, spatial, act, a, as_stream(stream), &launched, what, &cv)));
    if (!launched && !cluster_disabled())
        DNB_TRY((run_cluster<false, false>(batch, filters, spatial, act, a, as_stream(stream), &launched, what, &cv)));
    if (!launched && !stage_disabled())
        DNB_TRY((run_stage<false, false>(batch, filters, spatial, act, a, as_stream(stream), &launched, what, &cv)));
    if (!launched) return fail(DNB_ERR_UNSUPPORTED, "%s: shape not taken by the fused kernel", what);
    return DNB_OK;
}

dnb_status dnb_syncbn_act_backward(dnb_comm comm, const float *x, const float *y, const float *delta, float *dx,
                                   int64_t batch, int64_t filters, int64_t spatial, const float *scales,
                                   const float *biases, const float *mean, const float *variance,
                                   float *bias_updates, float *scale_updates, float *mean_delta,
                                   float *variance_delta, int act, dnb_stream stream) {
    const char *what = "syncbn_act_backward";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (filters == 0) return DNB_OK;
    if (!x || !delta || !dx || !scales || !biases || !mean || !variance || !bias_updates || !scale_updates ||
        !mean_delta || !variance_delta)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    CommView cv;
    DNB_TRY(comm_next(comm, &cv));
    if (filters > cv.cmax) return fail(DNB_ERR_UNSUPPORTED, "%s: %lld channels, communicator holds %lld", what,
                                       (long long)filters, (long long)cv.cmax);
    if (!(aligned16(x) && aligned16(delta) && aligned16(dx) && (!y || aligned16(y))))
        return fail(DNB_ERR_UNSUPPORTED, "%s: tensors must be 16-byte aligned", what);
    BnIO a;
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
    bool launched = false;
    const cudaStream_t s = as_stream(stream);
    if (y)
        DNB_TRY((run_sweep<true, true>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
    else
        DNB_TRY((run_sweep<true, false>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
    if (!launched && !cluster_disabled()) {
        if (y)
            DNB_TRY((run_cluster<true, true>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
        else
            DNB_TRY((run_cluster<true, false>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
    }
    if (!launched && !stage_disabled()) {
        if (y)
            DNB_TRY((run_stage<true, true>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
        else
            DNB_TRY((run_stage<true, false>(batch, filters, spatial, act, a, s, &launched, what, &cv)));
    }
    if (!launched) return fail(DNB_ERR_UNSUPPORTED, "%s: shape not taken by the fused kernel", what);
    return DNB_OK;
}

dnb_status dnb_bn_act_forward_from_stats(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                         int64_t spatial, const double *pieces, int64_t npieces,
                                         const float *scales, const float *biases, float *mean, float *variance,
                                         float *rolling_mean, float *rolling_variance, int act,
                                         dnb_stream stream) {
    const char *what = "bn_act_forward_from_stats";
    DNB_TRY(check_shape(batch, filters, spatial, what));
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "%s: unknown activation %d", what, act);
    if (npieces < 1) return fail(DNB_ERR_INVALID, "%s: npieces must be >= 1", what);
    if (filters == 0) return DNB_OK;
    if (!x || !y || !pieces || !scales || !biases || !mean || !variance || !rolling_mean || !rolling_variance)
        return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    const cudaStream_t s = as_stream(stream);
    const GGeom g = make_ggeom(batch, filters, spatial, aligned16(x));
    Workspace *ws = nullptr;
    DNB_TRY(workspace(s, GScratch::bytes(g), &ws));
    const GScratch sc = GScratch::carve(ws->scratch, g);
    float4 *tab = static_cast<float4 *>(sc.tab);
    k_fwd_finalize_pieces<<<(unsigned)((filters + kPieceCh - 1) / kPieceCh), kPieceCh * kPieceSlices, 0, s>>>(
        filters, npieces, pieces, scales, biases, mean, variance, rolling_mean, rolling_variance, tab);
    DNB_TRY(after_launch(s, what));
    const bool al = aligned16(x) && aligned16(y) && (!x_norm || aligned16(x_norm));
    return dispatch_act(act, [&]<int A>() {
        return chan::launch_chan(batch, filters, spatial, OpFwdApply<A>{x, y, x_norm, tab, act, al}, s, what);
    });
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
