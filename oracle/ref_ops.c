/*
 * TEST INFRASTRUCTURE -- the CPU oracle. Nothing in the product links this file.
 *
 * A C restatement of darknet-zig's CPU array ops for the elementwise / reduction /
 * broadcast path: src/blas.zig, src/activations.zig, the pooling loops of
 * src/layers/pooling.zig, the op sequences of src/layers/batchnorm.zig and the SGD
 * update of src/layers/convolutional.zig. Every function names the reference lines it
 * follows and keeps the reference's loop order and float operation order, so that a
 * bit-exact comparison against it is meaningful.
 *
 * Float semantics (Zig -> C):
 *   - the whole file is built with -ffp-contract=off and without -ffast-math: Zig's
 *     default "strict" float mode never fuses a*b+c;
 *   - axpy runs under @setFloatMode(.optimized) (blas.zig:21-24), which lets LLVM fuse
 *     the multiply-add; on an FMA-capable host that is a single rounding, so axpy is
 *     restated with fmaf();
 *   - @exp/@log/@sqrt are libm expf/logf/sqrtf; std.math.pow(f32, v, -1.5) is Zig
 *     standard-library code that is not part of the reference tree, restated as powf
 *     (ulp-level differences are covered by the reduction tolerance).
 *
 * Threading: the reference ops are single-threaded loops. oracle_set_threads(n>1)
 * splits the OUTER loop of each op (channels for per-channel reductions, planes or
 * element ranges for elementwise work) across OpenMP threads. Every output element is
 * still produced by one thread in the reference's order, so results are bit-identical
 * to the single-threaded run; only the timed CPU baseline uses it.
 */
#include <float.h>
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#include "ref_ops.h"

static int g_threads = 1;

void oracle_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
int oracle_get_threads(void) { return g_threads; }

/* Zig folds `1.0507 * 1.6732` at comptime in extended precision and rounds the product
 * to f32 once (activations.zig:65,95); two f32 literals multiplied in float would round
 * three times. */
#define SELU_SCALE_ALPHA ((float)(1.0507 * 1.6732))

#define PAR_FOR _Pragma("omp parallel for schedule(static) num_threads(g_threads) if(g_threads > 1)")

/* ------------------------------------------------------------------------- */
/* blas.zig:13-46 -- vector ops                                               */
/* ------------------------------------------------------------------------- */

/* blas.zig:13-15 */
void ref_fill(float *x, int64_t n, float alpha) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) x[i] = alpha;
}

/* blas.zig:17-19 */
void ref_copy(const float *src, float *dst, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) dst[i] = src[i];
}

/* blas.zig:21-24 (optimized float mode: the multiply-add is fused) */
void ref_axpy(float alpha, const float *x, float *y, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) y[i] = fmaf(alpha, x[i], y[i]);
}

/* blas.zig:26-29 */
void ref_scal(float alpha, float *x, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] * alpha;
}

/* blas.zig:31-33 */
void ref_mul(const float *x, float *y, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) y[i] = y[i] * x[i];
}

/* darknet_kernels.hip:150-153 add_scalar_kernel; it has no CPU twin, so the oracle is
 * the strict single-rounding add. */
void ref_add_scalar(float alpha, float *x, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) x[i] = x[i] + alpha;
}

/* blas.zig:44-46: std.math.clamp(v, -a, a) == @max(-a, @min(v, a)) */
void ref_constrain(float alpha, float *x, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) {
        float v = x[i];
        float lo = v < alpha ? v : alpha;
        x[i] = lo > -alpha ? lo : -alpha;
    }
}

/* ------------------------------------------------------------------------- */
/* activations.zig                                                            */
/* ------------------------------------------------------------------------- */

/* activations.zig:58-82, one element; enum numbering activations.zig:11-27 */
float ref_activate(float x, int a) {
    switch (a) {
    case ACT_LINEAR: return x;
    case ACT_LOGISTIC: return 1.0f / (1.0f + expf(-x));
    case ACT_LOGGY: return 2.0f / (1.0f + expf(-x)) - 1.0f;
    case ACT_RELU: return x > 0 ? x : 0.0f;
    case ACT_ELU: return x >= 0 ? x : expf(x) - 1.0f;
    case ACT_SELU: return x >= 0 ? 1.0507f * x : SELU_SCALE_ALPHA * (expf(x) - 1.0f);
    case ACT_RELIE: return x > 0 ? x : 0.01f * x;
    case ACT_RAMP: return (x > 0 ? x : 0.0f) + 0.1f * x;
    case ACT_LEAKY: return x > 0 ? x : 0.1f * x;
    case ACT_TANH: {
        float e = expf(2.0f * x);
        return (e - 1.0f) / (e + 1.0f);
    }
    case ACT_PLSE:
        if (x < -4.0f) return 0.01f * (x + 4.0f);
        if (x > 4.0f) return 0.01f * (x - 4.0f) + 1.0f;
        return 0.125f * x + 0.5f;
    case ACT_STAIR: {
        float n = floorf(x);
        int64_t ni = (int64_t)n;
        /* Zig @rem keeps the dividend's sign, as C's % does */
        if (ni % 2 == 0) return floorf(x / 2.0f);
        return (x - n) + floorf(x / 2.0f);
    }
    case ACT_HARDTAN: {
        float lo = x < 1.0f ? x : 1.0f;
        return lo > -1.0f ? lo : -1.0f;
    }
    case ACT_LHTAN:
        if (x < 0) return 0.001f * x;
        if (x > 1.0f) return 0.001f * (x - 1.0f) + 1.0f;
        return x;
    }
    return 0.0f;
}

/* activations.zig:85-105; y is the activation OUTPUT */
float ref_gradient(float y, int a) {
    switch (a) {
    case ACT_LINEAR: return 1.0f;
    case ACT_LOGISTIC: return (1.0f - y) * y;
    case ACT_LOGGY: {
        float t = (y + 1.0f) / 2.0f;
        return 2.0f * (1.0f - t) * t;
    }
    case ACT_RELU: return y > 0 ? 1.0f : 0.0f;
    case ACT_ELU: return y >= 0 ? 1.0f : y + 1.0f;
    case ACT_SELU: return y >= 0 ? 1.0507f : y + SELU_SCALE_ALPHA;
    case ACT_RELIE: return y > 0 ? 1.0f : 0.01f;
    case ACT_RAMP: return (y > 0 ? 1.0f : 0.0f) + 0.1f;
    case ACT_LEAKY: return y > 0 ? 1.0f : 0.1f;
    case ACT_TANH: return 1.0f - y * y;
    case ACT_PLSE: return (y < 0 || y > 1.0f) ? 0.01f : 0.125f;
    case ACT_STAIR: return floorf(y) == y ? 0.0f : 1.0f;
    case ACT_HARDTAN: return (y > -1.0f && y < 1.0f) ? 1.0f : 0.0f;
    case ACT_LHTAN: return (y > 0 && y < 1.0f) ? 1.0f : 0.001f;
    }
    return 0.0f;
}

/* activations.zig:107-125 (the hoisted fast paths are what runs for leaky/relu/logistic) */
void ref_activate_array(float *x, int64_t n, int a) {
    if (a == ACT_LINEAR) return;
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) x[i] = ref_activate(x[i], a);
}

/* activations.zig:127-143: delta *= gradient(y) */
void ref_gradient_array(const float *y, int64_t n, int a, float *delta) {
    if (a == ACT_LINEAR) return;
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) delta[i] = delta[i] * ref_gradient(y[i], a);
}

/* ------------------------------------------------------------------------- */
/* blas.zig:53-100 -- bias / scale, NCHW output[((b*filters)+f)*spatial+s]     */
/* ------------------------------------------------------------------------- */

/* blas.zig:53-61 */
void ref_add_bias(float *out, const float *biases, int64_t batch, int64_t filters, int64_t spatial) {
    PAR_FOR
    for (int64_t p = 0; p < batch * filters; ++p) {
        float bias = biases[p % filters];
        float *row = out + p * spatial;
        for (int64_t s = 0; s < spatial; ++s) row[s] = row[s] + bias;
    }
}

/* blas.zig:63-71 */
void ref_scale_bias(float *out, const float *scales, int64_t batch, int64_t filters, int64_t spatial) {
    PAR_FOR
    for (int64_t p = 0; p < batch * filters; ++p) {
        float sc = scales[p % filters];
        float *row = out + p * spatial;
        for (int64_t s = 0; s < spatial; ++s) row[s] = row[s] * sc;
    }
}

/* blas.zig:73-82: one sum per plane, added to bias_updates[f] in batch order. The
 * loops are swapped (f outer) so threads own channels; each bias_updates[f] still
 * receives its planes in b order. */
void ref_backward_bias(float *bias_updates, const float *delta, int64_t batch, int64_t filters, int64_t spatial) {
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        for (int64_t b = 0; b < batch; ++b) {
            const float *row = delta + (b * filters + f) * spatial;
            float sum = 0.0f;
            for (int64_t s = 0; s < spatial; ++s) sum += row[s];
            bias_updates[f] += sum;
        }
    }
}

/* blas.zig:84-100: one accumulator per channel over (b, s) */
void ref_backward_scale(const float *x_norm, const float *delta, int64_t batch, int64_t filters, int64_t spatial,
                        float *scale_updates) {
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        float sum = 0.0f;
        for (int64_t b = 0; b < batch; ++b) {
            const int64_t base = (b * filters + f) * spatial;
            for (int64_t s = 0; s < spatial; ++s) sum += delta[base + s] * x_norm[base + s];
        }
        scale_updates[f] += sum;
    }
}

/* ------------------------------------------------------------------------- */
/* blas.zig:106-204 -- batch normalisation                                    */
/* ------------------------------------------------------------------------- */

/* blas.zig:106-116 */
void ref_mean(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out) {
    const float scale_f = 1.0f / (float)(batch * spatial);
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        float sum = 0.0f;
        for (int64_t b = 0; b < batch; ++b) {
            const float *row = x + (b * filters + f) * spatial;
            for (int64_t s = 0; s < spatial; ++s) sum += row[s];
        }
        out[f] = sum * scale_f;
    }
}

/* blas.zig:121-135: unbiased (batch*spatial - 1) */
void ref_variance(const float *x, const float *mean, int64_t batch, int64_t filters, int64_t spatial, float *out) {
    const float scale_f = 1.0f / (float)(batch * spatial - 1);
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        float sum = 0.0f;
        const float m = mean[f];
        for (int64_t b = 0; b < batch; ++b) {
            const float *row = x + (b * filters + f) * spatial;
            for (int64_t s = 0; s < spatial; ++s) {
                float d = row[s] - m;
                sum += d * d;
            }
        }
        out[f] = sum * scale_f;
    }
}

/* blas.zig:137-146: multiply by 1/(sqrt(var)+1e-6) */
void ref_normalize(float *x, const float *mean, const float *variance, int64_t batch, int64_t filters,
                   int64_t spatial) {
    PAR_FOR
    for (int64_t p = 0; p < batch * filters; ++p) {
        const int64_t f = p % filters;
        const float m = mean[f];
        const float inv = 1.0f / (sqrtf(variance[f]) + 0.000001f);
        float *row = x + p * spatial;
        for (int64_t s = 0; s < spatial; ++s) row[s] = (row[s] - m) * inv;
    }
}

/* blas.zig:148-157 */
void ref_mean_delta(const float *delta, const float *variance, int64_t batch, int64_t filters, int64_t spatial,
                    float *out) {
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        float sum = 0.0f;
        for (int64_t b = 0; b < batch; ++b) {
            const float *row = delta + (b * filters + f) * spatial;
            for (int64_t s = 0; s < spatial; ++s) sum += row[s];
        }
        out[f] = sum * (-1.0f / sqrtf(variance[f] + 0.00001f));
    }
}

/* blas.zig:159-178 */
void ref_variance_delta(const float *x, const float *delta, const float *mean, const float *variance, int64_t batch,
                        int64_t filters, int64_t spatial, float *out) {
    PAR_FOR
    for (int64_t f = 0; f < filters; ++f) {
        float sum = 0.0f;
        const float m = mean[f];
        for (int64_t b = 0; b < batch; ++b) {
            const int64_t base = (b * filters + f) * spatial;
            for (int64_t s = 0; s < spatial; ++s) sum += delta[base + s] * (x[base + s] - m);
        }
        out[f] = sum * -0.5f * powf(variance[f] + 0.00001f, -1.5f);
    }
}

/* blas.zig:180-204 */
void ref_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                         const float *variance_delta, int64_t batch, int64_t filters, int64_t spatial, float *delta) {
    const float denom = (float)(spatial * batch);
    PAR_FOR
    for (int64_t p = 0; p < batch * filters; ++p) {
        const int64_t f = p % filters;
        const float inv = 1.0f / sqrtf(variance[f] + 0.00001f);
        const float vd = variance_delta[f];
        const float md = mean_delta[f];
        const float m = mean[f];
        float *drow = delta + p * spatial;
        const float *xrow = x + p * spatial;
        for (int64_t s = 0; s < spatial; ++s)
            drow[s] = drow[s] * inv + vd * 2.0f * (xrow[s] - m) / denom + md / denom;
    }
}

/* ------------------------------------------------------------------------- */
/* blas.zig:213-252 -- softmax and cross entropy                              */
/* ------------------------------------------------------------------------- */

/* blas.zig:213-223 */
static void softmax_one(const float *in, int64_t n, float temp, int64_t stride, float *out) {
    float largest = -FLT_MAX;
    for (int64_t i = 0; i < n; ++i) {
        float v = in[i * stride];
        largest = v > largest ? v : largest;
    }
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) {
        float e = expf(in[i * stride] / temp - largest / temp);
        sum += e;
        out[i * stride] = e;
    }
    for (int64_t i = 0; i < n; ++i) out[i * stride] = out[i * stride] / sum;
}

/* blas.zig:225-242 */
void ref_softmax(const float *input, int64_t n, int64_t batch, int64_t batch_offset, int64_t groups,
                 int64_t group_offset, int64_t stride, float temp, float *output) {
    PAR_FOR
    for (int64_t q = 0; q < batch * groups; ++q) {
        const int64_t b = q / groups, g = q % groups;
        const int64_t off = b * batch_offset + g * group_offset;
        softmax_one(input + off, n, temp, stride, output + off);
    }
}

/* blas.zig:247-252 (the CPU path does not clamp p before the log) */
void ref_softmax_cross_entropy(const float *pred, const float *truth, float *delta, float *err, int64_t n) {
    PAR_FOR
    for (int64_t i = 0; i < n; ++i) {
        const float t = truth[i], p = pred[i];
        err[i] = t != 0.0f ? -logf(p) : 0.0f;
        delta[i] = t - p;
    }
}

/* utils.zig:71-75 -- the host-side loss sum after softmax_x_ent (misc.zig:48-49) */
float ref_sum_array(const float *a, int64_t n) {
    float sum = 0.0f;
    for (int64_t i = 0; i < n; ++i) sum += a[i];
    return sum;
}

/* ------------------------------------------------------------------------- */
/* blas.zig:290-322 -- shortcut                                                */
/* ------------------------------------------------------------------------- */
void ref_shortcut(int64_t batch, int64_t w1, int64_t h1, int64_t c1, const float *add, int64_t w2, int64_t h2,
                  int64_t c2, float s1, float s2, float *out) {
    int64_t stride = w1 / w2, sample = w2 / w1;
    if (stride < 1) stride = 1;
    if (sample < 1) sample = 1;
    const int64_t minw = w1 < w2 ? w1 : w2;
    const int64_t minh = h1 < h2 ? h1 : h2;
    const int64_t minc = c1 < c2 ? c1 : c2;
    PAR_FOR
    for (int64_t q = 0; q < batch * minc; ++q) {
        const int64_t b = q / minc, k = q % minc;
        for (int64_t j = 0; j < minh; ++j) {
            for (int64_t i = 0; i < minw; ++i) {
                const int64_t oi = i * sample + w2 * (j * sample + h2 * (k + c2 * b));
                const int64_t ai = i * stride + w1 * (j * stride + h1 * (k + c1 * b));
                out[oi] = s1 * out[oi] + s2 * add[ai];
            }
        }
    }
}

/* ------------------------------------------------------------------------- */
/* layers/pooling.zig                                                         */
/* ------------------------------------------------------------------------- */

/* pooling.zig:33-34 */
int64_t ref_maxpool_out_dim(int64_t in, int64_t size, int64_t stride, int64_t pad) {
    return (in + pad - size) / stride + 1;
}

/* pooling.zig:59-93: offset -pad/2, taps outside the image are skipped, strict '>' so
 * the first maximum in (row, col) tap order wins, index = flat input index (or -1). */
void ref_forward_maxpool(int64_t batch, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride, int64_t size,
                         int64_t pad, const float *input, float *output, int32_t *indexes) {
    const int64_t off = -(pad / 2);
    const int64_t h = ref_maxpool_out_dim(in_h, size, stride, pad);
    const int64_t w = ref_maxpool_out_dim(in_w, size, stride, pad);
    PAR_FOR
    for (int64_t q = 0; q < batch * in_c; ++q) {
        const int64_t b = q / in_c, k = q % in_c;
        for (int64_t i = 0; i < h; ++i) {
            for (int64_t j = 0; j < w; ++j) {
                const int64_t out_index = j + w * (i + h * (k + in_c * b));
                float max = -FLT_MAX;
                int32_t max_i = -1;
                for (int64_t n = 0; n < size; ++n) {
                    for (int64_t m = 0; m < size; ++m) {
                        const int64_t cur_h = off + i * stride + n;
                        const int64_t cur_w = off + j * stride + m;
                        if (cur_h < 0 || cur_h >= in_h) continue;
                        if (cur_w < 0 || cur_w >= in_w) continue;
                        const int64_t index = cur_w + in_w * (cur_h + in_h * (k + b * in_c));
                        const float val = input[index];
                        if (val > max) {
                            max = val;
                            max_i = (int32_t)index;
                        }
                    }
                }
                output[out_index] = max;
                indexes[out_index] = max_i;
            }
        }
    }
}

/* pooling.zig:95-103: scatter-add of the output delta to the selected inputs */
void ref_backward_maxpool(int64_t out_n, const float *delta, const int32_t *indexes, float *prev_delta) {
    for (int64_t i = 0; i < out_n; ++i) {
        const int32_t index = indexes[i];
        if (index < 0) continue;
        prev_delta[index] += delta[i];
    }
}

/* pooling.zig:146-158 */
void ref_forward_avgpool(int64_t batch, int64_t c, int64_t h, int64_t w, const float *input, float *output) {
    const int64_t spatial = h * w;
    const float denom = (float)spatial;
    PAR_FOR
    for (int64_t q = 0; q < batch * c; ++q) {
        const float *row = input + spatial * q;
        float sum = 0.0f;
        for (int64_t s = 0; s < spatial; ++s) sum += row[s];
        output[q] = sum / denom;
    }
}

/* pooling.zig:160-172 */
void ref_backward_avgpool(int64_t batch, int64_t c, int64_t h, int64_t w, const float *out_delta, float *in_delta) {
    const int64_t spatial = h * w;
    const float denom = (float)spatial;
    PAR_FOR
    for (int64_t q = 0; q < batch * c; ++q) {
        const float d = out_delta[q] / denom;
        float *row = in_delta + spatial * q;
        for (int64_t s = 0; s < spatial; ++s) row[s] += d;
    }
}

/* ------------------------------------------------------------------------- */
/* layer sequences: the reference's op order composed from the functions above */
/* ------------------------------------------------------------------------- */

/* layers/batchnorm.zig:74-99 (conv with batch_normalize: output already holds the conv
 * result) followed by the activation pass of convolutional.zig:171.
 *   x          in : conv output (not modified)
 *   x_saved    out: l.x (copy of x), may be NULL
 *   x_norm     out: l.x_norm (train only), may be NULL
 *   y          out: activated output (l.output)
 * rolling_momentum = 0.99 (batchnorm.zig:16). */
void ref_bn_forward_layer(const float *x, float *y, float *x_saved, float *x_norm, int64_t batch, int64_t filters,
                          int64_t spatial, const float *scales, const float *biases, float *mean, float *variance,
                          float *rolling_mean, float *rolling_variance, int train, int act) {
    const int64_t n = batch * filters * spatial;
    const float momentum = 0.99f;
    ref_copy(x, y, n);
    if (x_saved) ref_copy(y, x_saved, n);
    if (train) {
        ref_mean(y, batch, filters, spatial, mean);
        ref_variance(y, mean, batch, filters, spatial, variance);
        ref_scal(momentum, rolling_mean, filters);
        ref_axpy(1.0f - momentum, mean, rolling_mean, filters);
        ref_scal(momentum, rolling_variance, filters);
        ref_axpy(1.0f - momentum, variance, rolling_variance, filters);
        ref_normalize(y, mean, variance, batch, filters, spatial);
        if (x_norm) ref_copy(y, x_norm, n);
    } else {
        ref_normalize(y, rolling_mean, rolling_variance, batch, filters, spatial);
    }
    ref_scale_bias(y, scales, batch, filters, spatial);
    ref_add_bias(y, biases, batch, filters, spatial);
    ref_activate_array(y, n, act);
}

/* convolutional.zig:178 (gradient) + layers/batchnorm.zig:101-118. delta is updated in
 * place into dL/dx. mean/variance are the batch statistics (train) or the rolling
 * ones (inference), exactly as batchnorm.zig:108-109 selects them. */
void ref_bn_backward_layer(const float *x, const float *x_norm, const float *y, float *delta, int64_t batch,
                           int64_t filters, int64_t spatial, const float *scales, const float *mean,
                           const float *variance, float *bias_updates, float *scale_updates, float *mean_delta,
                           float *variance_delta, int act) {
    const int64_t n = batch * filters * spatial;
    ref_gradient_array(y, n, act, delta);
    ref_backward_bias(bias_updates, delta, batch, filters, spatial);
    ref_backward_scale(x_norm, delta, batch, filters, spatial, scale_updates);
    ref_scale_bias(delta, scales, batch, filters, spatial);
    ref_mean_delta(delta, variance, batch, filters, spatial, mean_delta);
    ref_variance_delta(x, delta, mean, variance, batch, filters, spatial, variance_delta);
    ref_normalize_delta(x, mean, variance, mean_delta, variance_delta, batch, filters, spatial, delta);
}

/* convolutional.zig:217-233 (the weight part): decay folded into the update, then the
 * momentum step. learning_rate already includes learning_rate_scale. */
void ref_sgd_update(float *w, float *wu, int64_t n, float learning_rate, float momentum, float decay, int64_t batch) {
    const float b = (float)batch;
    ref_axpy(-decay * b, w, wu, n);
    ref_axpy(learning_rate / b, wu, w, n);
    ref_scal(momentum, wu, n);
}
