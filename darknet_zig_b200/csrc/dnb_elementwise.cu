// Elementwise and per-channel broadcast ops: blas.zig:13-71, activations.zig:107-143,
// blas.zig:137-146 and :180-204 (normalize, normalize_delta), the SGD update of
// convolutional.zig:217-233 and the same-shape shortcut of blas.zig:290-322.
//
// Every op reads and writes each element once with 128-bit accesses when the pointers
// are 16-byte aligned (a scalar tail covers n % 4), so each is bound by HBM bandwidth at
// its compulsory bytes per element. Arithmetic is bit-identical to the reference CPU
// ops: --fmad=false keeps a*b+c as two roundings, and __fmaf_rn appears exactly where
// blas.axpy fuses.
#include "dnb_cdiv.cuh"
#include "dnb_chan.cuh"

namespace dnb {
namespace {

using chan::kThreads;
using chan::kUnroll;
using chan::launch_chan;

// Grid-stride driver. Op supplies: bool vec (all of its arrays are 16-byte aligned),
// V load(i4) / void store(i4, V) for float4 index i4, void scalar(i) for element i.
// The tile loop issues kUnroll independent loads per thread before any store.
template <class Op>
__global__ void __launch_bounds__(kThreads) k_map(int64_t n, Op op) {
    const int64_t n4 = op.vec ? (n >> 2) : 0;
    const int64_t tile = (int64_t)kThreads * kUnroll;
    for (int64_t base = (int64_t)blockIdx.x * tile; base < n4; base += (int64_t)gridDim.x * tile) {
        typename Op::V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads + threadIdx.x;
            if (i < n4) v[u] = op.load(i);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads + threadIdx.x;
            if (i < n4) op.store(i, v[u]);
        }
    }
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t j = (n4 << 2) + (int64_t)blockIdx.x * kThreads + threadIdx.x; j < n; j += step) op.scalar(j);
}

template <class Op>
dnb_status launch_map(int64_t n, const Op &op, cudaStream_t stream, const char *what) {
    if (n < 0) return fail(DNB_ERR_INVALID, "%s: negative size", what);
    if (n == 0) return DNB_OK;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const int64_t items = op.vec ? ((n >> 2) + kUnroll - 1) / kUnroll : n;
    k_map<Op><<<grid_for(items, kThreads, ds), kThreads, 0, stream>>>(n, op);
    return after_launch(stream, what);
}

// ---- blas.zig:13-46 ----
struct OpFill {
    float *x;
    float a;
    bool vec;
    struct V {};
    __device__ V load(int64_t) const { return {}; }
    __device__ void store(int64_t i, V) const { st4(x + 4 * i, make_float4(a, a, a, a)); }
    __device__ void scalar(int64_t i) const { x[i] = a; }
};

struct OpCopy {
    const float *x;
    float *y;
    bool vec;
    using V = float4;
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ void store(int64_t i, V v) const { st4(y + 4 * i, v); }
    __device__ void scalar(int64_t i) const { y[i] = x[i]; }
};

struct OpAxpy {  // y = fma(a, x, y), blas.zig:21-24
    const float *x;
    float *y;
    float a;
    bool vec;
    struct V { float4 x, y; };
    __device__ V load(int64_t i) const { return {ld4(x + 4 * i), ld4(y + 4 * i)}; }
    __device__ void store(int64_t i, V v) const {
        st4(y + 4 * i, make_float4(__fmaf_rn(a, v.x.x, v.y.x), __fmaf_rn(a, v.x.y, v.y.y), __fmaf_rn(a, v.x.z, v.y.z),
                                   __fmaf_rn(a, v.x.w, v.y.w)));
    }
    __device__ void scalar(int64_t i) const { y[i] = __fmaf_rn(a, x[i], y[i]); }
};

struct OpScal {
    float *x;
    float a;
    bool vec;
    using V = float4;
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ void store(int64_t i, V v) const { st4(x + 4 * i, make_float4(v.x * a, v.y * a, v.z * a, v.w * a)); }
    __device__ void scalar(int64_t i) const { x[i] = x[i] * a; }
};

struct OpMul {
    const float *x;
    float *y;
    bool vec;
    struct V { float4 x, y; };
    __device__ V load(int64_t i) const { return {ld4(x + 4 * i), ld4(y + 4 * i)}; }
    __device__ void store(int64_t i, V v) const {
        st4(y + 4 * i, make_float4(v.y.x * v.x.x, v.y.y * v.x.y, v.y.z * v.x.z, v.y.w * v.x.w));
    }
    __device__ void scalar(int64_t i) const { y[i] = y[i] * x[i]; }
};

struct OpAddScalar {
    float *x;
    float a;
    bool vec;
    using V = float4;
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ void store(int64_t i, V v) const { st4(x + 4 * i, make_float4(v.x + a, v.y + a, v.z + a, v.w + a)); }
    __device__ void scalar(int64_t i) const { x[i] = x[i] + a; }
};

// std.math.clamp(v, -a, a) == max(-a, min(v, a)) (blas.zig:44-46)
__device__ __forceinline__ float clampf(float v, float a) {
    float lo = v < a ? v : a;
    return lo > -a ? lo : -a;
}
struct OpConstrain {
    float *x;
    float a;
    bool vec;
    using V = float4;
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ void store(int64_t i, V v) const {
        st4(x + 4 * i, make_float4(clampf(v.x, a), clampf(v.y, a), clampf(v.z, a), clampf(v.w, a)));
    }
    __device__ void scalar(int64_t i) const { x[i] = clampf(x[i], a); }
};

// ---- activations.zig:107-143 ----
template <int A>
struct OpActivate {
    float *x;
    int act;
    bool vec;
    using V = float4;
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ void store(int64_t i, V v) const {
        st4(x + 4 * i, make_float4(act_fwd<A>(v.x, act), act_fwd<A>(v.y, act), act_fwd<A>(v.z, act),
                                   act_fwd<A>(v.w, act)));
    }
    __device__ void scalar(int64_t i) const { x[i] = act_fwd<A>(x[i], act); }
};

template <int A>
struct OpGradient {  // delta *= gradient(y)
    const float *y;
    float *d;
    int act;
    bool vec;
    struct V { float4 y, d; };
    __device__ V load(int64_t i) const { return {ld4(y + 4 * i), ld4(d + 4 * i)}; }
    __device__ void store(int64_t i, V v) const {
        st4(d + 4 * i, make_float4(v.d.x * act_grad<A>(v.y.x, act), v.d.y * act_grad<A>(v.y.y, act),
                                   v.d.z * act_grad<A>(v.y.z, act), v.d.w * act_grad<A>(v.y.w, act)));
    }
    __device__ void scalar(int64_t i) const { d[i] = d[i] * act_grad<A>(y[i], act); }
};

// ---- SGD: convolutional.zig:230-232 / 332-334 fused ----
__device__ __forceinline__ void sgd1(float &w, float &wu, float a_decay, float a_lr, float mom) {
    wu = __fmaf_rn(a_decay, w, wu);  // axpy(-decay*batch, w, wu)
    w = __fmaf_rn(a_lr, wu, w);      // axpy(lr/batch, wu, w)
    wu = wu * mom;                   // scal(momentum, wu)
}
struct OpSgd {
    float *w, *wu;
    float a_decay, a_lr, mom;
    bool vec;
    struct V { float4 w, u; };
    __device__ V load(int64_t i) const { return {ld4(w + 4 * i), ld4(wu + 4 * i)}; }
    __device__ void store(int64_t i, V v) const {
        sgd1(v.w.x, v.u.x, a_decay, a_lr, mom);
        sgd1(v.w.y, v.u.y, a_decay, a_lr, mom);
        sgd1(v.w.z, v.u.z, a_decay, a_lr, mom);
        sgd1(v.w.w, v.u.w, a_decay, a_lr, mom);
        st4(w + 4 * i, v.w);
        st4(wu + 4 * i, v.u);
    }
    __device__ void scalar(int64_t i) const {
        float a = w[i], b = wu[i];
        sgd1(a, b, a_decay, a_lr, mom);
        w[i] = a;
        wu[i] = b;
    }
};

// ---- shortcut, same shape (blas.zig:317 with stride = sample = 1) ----
struct OpShortcutSame {
    const float *add;
    float *out;
    float s1, s2;
    bool vec;
    struct V { float4 o, a; };
    __device__ V load(int64_t i) const { return {ld4(out + 4 * i), ld4(add + 4 * i)}; }
    __device__ void store(int64_t i, V v) const {
        st4(out + 4 * i, make_float4(s1 * v.o.x + s2 * v.a.x, s1 * v.o.y + s2 * v.a.y, s1 * v.o.z + s2 * v.a.z,
                                     s1 * v.o.w + s2 * v.a.w));
    }
    __device__ void scalar(int64_t i) const { out[i] = s1 * out[i] + s2 * add[i]; }
};

// General shortcut with resampling (blas.zig:290-322): one thread per (b, k, j, i).
__global__ void k_shortcut_general(int64_t size, int64_t minw, int64_t minh, int64_t minc, int64_t stride,
                                   int64_t sample, int64_t w1, int64_t h1, int64_t c1, const float *add, int64_t w2,
                                   int64_t h2, int64_t c2, float s1, float s2, float *out) {
    for (int64_t id = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; id < size;
         id += (int64_t)gridDim.x * blockDim.x) {
        int64_t t = id;
        const int64_t i = t % minw;
        t /= minw;
        const int64_t j = t % minh;
        t /= minh;
        const int64_t k = t % minc;
        const int64_t b = t / minc;
        const int64_t oi = i * sample + w2 * (j * sample + h2 * (k + c2 * b));
        const int64_t ai = i * stride + w1 * (j * stride + h1 * (k + c1 * b));
        out[oi] = s1 * out[oi] + s2 * add[ai];
    }
}

// blas.zig:53-61
struct OpAddBias {
    float *out;
    const float *b;
    bool vec;
    using P = float;
    using V = float4;
    __device__ P param(int64_t c) const { return b[c]; }
    __device__ V load(int64_t i) const { return ld4(out + 4 * i); }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        st4(out + 4 * i, make_float4(v.x + p0, v.y + p1, v.z + p2, v.w + p3));
    }
    __device__ void scalar(int64_t i, P p) const { out[i] = out[i] + p; }
};

// blas.zig:63-71
struct OpScaleBias {
    float *out;
    const float *s;
    bool vec;
    using P = float;
    using V = float4;
    __device__ P param(int64_t c) const { return s[c]; }
    __device__ V load(int64_t i) const { return ld4(out + 4 * i); }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        st4(out + 4 * i, make_float4(v.x * p0, v.y * p1, v.z * p2, v.w * p3));
    }
    __device__ void scalar(int64_t i, P p) const { out[i] = out[i] * p; }
};

// blas.zig:137-146: (x - m) * (1/(sqrt(v) + 1e-6))
struct OpNormalize {
    float *x;
    const float *mean, *var;
    bool vec;
    using P = float2;  // (mean, inv)
    using V = float4;
    __device__ P param(int64_t c) const { return make_float2(mean[c], 1.0f / (sqrtf(var[c]) + 0.000001f)); }
    __device__ V load(int64_t i) const { return ld4(x + 4 * i); }
    __device__ static float f(float v, P p) { return (v - p.x) * p.y; }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        st4(x + 4 * i, make_float4(f(v.x, p0), f(v.y, p1), f(v.z, p2), f(v.w, p3)));
    }
    __device__ void scalar(int64_t i, P p) const { x[i] = f(x[i], p); }
};

// blas.zig:180-204: d*inv + vd*2*(x-m)/denom + md/denom
struct NDParam {
    float inv, vd, md_over, m;
};
// the division by the element count is done by the launch's ConstDiv (dnb_cdiv.cuh)
__device__ __forceinline__ float norm_delta_num(float x, const NDParam &p) { return p.vd * 2.0f * (x - p.m); }
__device__ __forceinline__ float norm_delta1(float d, const NDParam &p, float q) { return d * p.inv + q + p.md_over; }
struct OpNormalizeDelta {
    const float *x, *mean, *var, *md, *vd;
    float *d;
    float denom;
    ConstDiv cdiv;
    bool vec;
    using P = NDParam;
    struct V { float4 d, x; };
    __device__ P param(int64_t c) const {
        NDParam p;
        p.inv = 1.0f / sqrtf(var[c] + 0.00001f);
        p.vd = vd[c];
        p.md_over = md[c] / denom;
        p.m = mean[c];
        return p;
    }
    __device__ V load(int64_t i) const { return {ld4(d + 4 * i), ld4(x + 4 * i)}; }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        const float4 q = div4_const(make_float4(norm_delta_num(v.x.x, p0), norm_delta_num(v.x.y, p1),
                                                norm_delta_num(v.x.z, p2), norm_delta_num(v.x.w, p3)),
                                    cdiv);
        st4(d + 4 * i, make_float4(norm_delta1(v.d.x, p0, q.x), norm_delta1(v.d.y, p1, q.y),
                                   norm_delta1(v.d.z, p2, q.z), norm_delta1(v.d.w, p3, q.w)));
    }
    __device__ void scalar(int64_t i, P p) const { d[i] = norm_delta1(d[i], p, div_const(norm_delta_num(x[i], p), cdiv)); }
};

// Inference BN + activation (batchnorm.zig:147-152 + convolutional.zig:269):
// act(((x - rm) * (1/(sqrt(rv)+1e-6))) * scale + bias)
struct BNParam {
    float m, inv, g, b;
};
template <int A>
struct OpBnInfer {
    const float *x;
    float *y;
    const float *rm, *rv, *g, *b;
    int act;
    bool vec;
    using P = BNParam;
    using V = float4;
    __device__ P param(int64_t c) const {
        BNParam p;
        p.m = rm[c];
        p.inv = 1.0f / (sqrtf(rv[c]) + 0.000001f);
        p.g = g[c];
        p.b = b[c];
        return p;
    }
    __device__ static float f(float v, const P &p, int act) { return act_fwd<A>((v - p.m) * p.inv * p.g + p.b, act); }
    __device__ V load(int64_t i) const { return ld4_stream(x + 4 * i); }
    __device__ void store(int64_t i, V v, P p0, P p1, P p2, P p3) const {
        st4(y + 4 * i, make_float4(f(v.x, p0, act), f(v.y, p1, act), f(v.z, p2, act), f(v.w, p3, act)));
    }
    __device__ void scalar(int64_t i, P p) const { y[i] = f(x[i], p, act); }
};

// pooling.zig:160-172: in_delta[q*S + s] += out_delta[q] / S (q = plane)
__global__ void __launch_bounds__(kThreads) k_avgpool_back(int64_t n, int64_t spatial, FastDiv fs, bool fast,
                                                          float *in_delta, const float *out_delta, float denom) {
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t j = (int64_t)blockIdx.x * kThreads + threadIdx.x; j < n; j += step) {
        const int64_t q = fast ? (int64_t)fs.div((uint32_t)j) : j / spatial;
        in_delta[j] = in_delta[j] + out_delta[q] / denom;
    }
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_fill(float *x, int64_t n, float alpha, dnb_stream stream) {
    if (n > 0 && !x) return fail(DNB_ERR_INVALID, "fill: x is null");
    return launch_map(n, OpFill{x, alpha, aligned16(x)}, as_stream(stream), "fill");
}

dnb_status dnb_copy(int64_t n, const float *x, float *y, dnb_stream stream) {
    if (n > 0 && (!x || !y)) return fail(DNB_ERR_INVALID, "copy: null pointer");
    return launch_map(n, OpCopy{x, y, aligned16(x) && aligned16(y)}, as_stream(stream), "copy");
}

dnb_status dnb_axpy(int64_t n, float alpha, const float *x, float *y, dnb_stream stream) {
    if (n > 0 && (!x || !y)) return fail(DNB_ERR_INVALID, "axpy: null pointer");
    return launch_map(n, OpAxpy{x, y, alpha, aligned16(x) && aligned16(y)}, as_stream(stream), "axpy");
}

dnb_status dnb_scal(int64_t n, float alpha, float *x, dnb_stream stream) {
    if (n > 0 && !x) return fail(DNB_ERR_INVALID, "scal: x is null");
    return launch_map(n, OpScal{x, alpha, aligned16(x)}, as_stream(stream), "scal");
}

dnb_status dnb_mul(int64_t n, const float *x, float *y, dnb_stream stream) {
    if (n > 0 && (!x || !y)) return fail(DNB_ERR_INVALID, "mul: null pointer");
    return launch_map(n, OpMul{x, y, aligned16(x) && aligned16(y)}, as_stream(stream), "mul");
}

dnb_status dnb_add_scalar(int64_t n, float alpha, float *x, dnb_stream stream) {
    if (n > 0 && !x) return fail(DNB_ERR_INVALID, "add_scalar: x is null");
    return launch_map(n, OpAddScalar{x, alpha, aligned16(x)}, as_stream(stream), "add_scalar");
}

dnb_status dnb_constrain(int64_t n, float alpha, float *x, dnb_stream stream) {
    if (n > 0 && !x) return fail(DNB_ERR_INVALID, "constrain: x is null");
    return launch_map(n, OpConstrain{x, alpha, aligned16(x)}, as_stream(stream), "constrain");
}

dnb_status dnb_activate_array(float *x, int64_t n, int act, dnb_stream stream) {
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "activate: unknown activation %d", act);
    if (act == DNB_ACT_LINEAR) return DNB_OK;  // activations.zig:111
    if (n > 0 && !x) return fail(DNB_ERR_INVALID, "activate: x is null");
    const cudaStream_t s = as_stream(stream);
    return dispatch_act(act, [&]<int A>() {
        return launch_map(n, OpActivate<A>{x, act, aligned16(x)}, s, "activate_array");
    });
}

dnb_status dnb_gradient_array(const float *y, int64_t n, int act, float *delta, dnb_stream stream) {
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "gradient: unknown activation %d", act);
    if (act == DNB_ACT_LINEAR) return DNB_OK;  // activations.zig:129
    if (n > 0 && (!y || !delta)) return fail(DNB_ERR_INVALID, "gradient: null pointer");
    const cudaStream_t s = as_stream(stream);
    return dispatch_act(act, [&]<int A>() {
        return launch_map(n, OpGradient<A>{y, delta, act, aligned16(y) && aligned16(delta)}, s, "gradient_array");
    });
}

dnb_status dnb_add_bias(float *output, const float *biases, int64_t batch, int64_t filters, int64_t spatial,
                        dnb_stream stream) {
    if (batch * filters * spatial > 0 && (!output || !biases)) return fail(DNB_ERR_INVALID, "add_bias: null pointer");
    return launch_chan(batch, filters, spatial, OpAddBias{output, biases, aligned16(output)}, as_stream(stream),
                       "add_bias");
}

dnb_status dnb_scale_bias(float *output, const float *scales, int64_t batch, int64_t filters, int64_t spatial,
                          dnb_stream stream) {
    if (batch * filters * spatial > 0 && (!output || !scales))
        return fail(DNB_ERR_INVALID, "scale_bias: null pointer");
    return launch_chan(batch, filters, spatial, OpScaleBias{output, scales, aligned16(output)}, as_stream(stream),
                       "scale_bias");
}

dnb_status dnb_normalize(float *x, const float *mean, const float *variance, int64_t batch, int64_t filters,
                         int64_t spatial, dnb_stream stream) {
    if (batch * filters * spatial > 0 && (!x || !mean || !variance))
        return fail(DNB_ERR_INVALID, "normalize: null pointer");
    return launch_chan(batch, filters, spatial, OpNormalize{x, mean, variance, aligned16(x)}, as_stream(stream),
                       "normalize");
}

dnb_status dnb_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                               const float *variance_delta, int64_t batch, int64_t filters, int64_t spatial,
                               float *delta, dnb_stream stream) {
    if (batch * filters * spatial > 0 && (!x || !mean || !variance || !mean_delta || !variance_delta || !delta))
        return fail(DNB_ERR_INVALID, "normalize_delta: null pointer");
    const float denom = (float)(spatial * batch);  // blas.zig:191
    OpNormalizeDelta op{x,     mean,  variance,        mean_delta, variance_delta,
                        delta, denom, const_div(denom), aligned16(x) && aligned16(delta)};
    return launch_chan(batch, filters, spatial, op, as_stream(stream), "normalize_delta");
}

dnb_status dnb_bn_act_forward_infer(const float *x, float *y, int64_t batch, int64_t filters, int64_t spatial,
                                    const float *scales, const float *biases, const float *rolling_mean,
                                    const float *rolling_variance, int act, dnb_stream stream) {
    if (!valid_act(act)) return fail(DNB_ERR_INVALID, "bn_act_forward_infer: unknown activation %d", act);
    if (batch * filters * spatial > 0 && (!x || !y || !scales || !biases || !rolling_mean || !rolling_variance))
        return fail(DNB_ERR_INVALID, "bn_act_forward_infer: null pointer");
    const cudaStream_t s = as_stream(stream);
    return dispatch_act(act, [&]<int A>() {
        OpBnInfer<A> op{x, y, rolling_mean, rolling_variance, scales, biases, act, aligned16(x) && aligned16(y)};
        return launch_chan(batch, filters, spatial, op, s, "bn_act_forward_infer");
    });
}

dnb_status dnb_sgd_momentum(int64_t n, float *weights, float *weight_updates, float learning_rate, float momentum,
                            float decay, int64_t batch, dnb_stream stream) {
    if (n > 0 && (!weights || !weight_updates)) return fail(DNB_ERR_INVALID, "sgd_momentum: null pointer");
    if (batch <= 0) return fail(DNB_ERR_INVALID, "sgd_momentum: batch must be positive");
    const float b = (float)batch;  // convolutional.zig:219
    OpSgd op{weights, weight_updates, -decay * b, learning_rate / b, momentum,
             aligned16(weights) && aligned16(weight_updates)};
    return launch_map(n, op, as_stream(stream), "sgd_momentum");
}

dnb_status dnb_shortcut(int64_t batch, int64_t w1, int64_t h1, int64_t c1, const float *add, int64_t w2, int64_t h2,
                        int64_t c2, float s1, float s2, float *out, dnb_stream stream) {
    if (batch < 0 || w1 <= 0 || h1 <= 0 || c1 <= 0 || w2 <= 0 || h2 <= 0 || c2 <= 0)
        return fail(DNB_ERR_INVALID, "shortcut: bad shape");
    if (batch == 0) return DNB_OK;
    if (!add || !out) return fail(DNB_ERR_INVALID, "shortcut: null pointer");
    const cudaStream_t s = as_stream(stream);
    if (w1 == w2 && h1 == h2 && c1 == c2) {
        const int64_t n = batch * w1 * h1 * c1;
        return launch_map(n, OpShortcutSame{add, out, s1, s2, aligned16(add) && aligned16(out)}, s, "shortcut");
    }
    int64_t stride = w1 / w2, sample = w2 / w1;  // gpu.zig:786-789
    if (stride < 1) stride = 1;
    if (sample < 1) sample = 1;
    const int64_t minw = w1 < w2 ? w1 : w2, minh = h1 < h2 ? h1 : h2, minc = c1 < c2 ? c1 : c2;
    const int64_t size = batch * minw * minh * minc;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    k_shortcut_general<<<grid_for(size, kThreads, ds), kThreads, 0, s>>>(size, minw, minh, minc, stride, sample, w1,
                                                                          h1, c1, add, w2, h2, c2, s1, s2, out);
    return after_launch(s, "shortcut");
}

dnb_status dnb_backward_avgpool(int64_t n, int64_t w, int64_t h, int64_t c, float *in_delta, const float *out_delta,
                                dnb_stream stream) {
    if (n < 0 || w <= 0 || h <= 0 || c <= 0) return fail(DNB_ERR_INVALID, "backward_avgpool: bad shape");
    if (n == 0) return DNB_OK;
    if (!in_delta || !out_delta) return fail(DNB_ERR_INVALID, "backward_avgpool: null pointer");
    const int64_t spatial = w * h, total = n * spatial;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const bool fast = total < (1ll << 32);
    const cudaStream_t s = as_stream(stream);
    k_avgpool_back<<<grid_for(total, kThreads, ds), kThreads, 0, s>>>(total, spatial, FastDiv((uint32_t)spatial), fast,
                                                                      in_delta, out_delta, (float)spatial);
    return after_launch(s, "backward_avgpool");
}

}  // extern "C"
