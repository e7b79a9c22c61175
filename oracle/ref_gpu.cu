// TEST INFRASTRUCTURE -- the reference's own device kernels, built for the B200.
//
// The reference kernel file (src/kernels/darknet_kernels.hip, path passed in as
// DNB_REFERENCE_KERNELS at build time) is #included unchanged and compiled by nvcc for
// sm_100a with the reference's flags (build.zig:144-156: `-x cu -O3`, nvcc's default
// floating-point contraction). Every ref_gpu_* entry point launches one of those kernels
// on the caller's stream with the grid the reference's dispatcher uses
// (src/gpu.zig:420-477): launch1d = ceil(n/256) blocks of 256 threads, launchPerFilter =
// one 256-thread block per filter.
//
// The two layer entries replay the reference's GPU layer sequences launch for launch:
//   ref_gpu_conv_bn_forward  convolutional.zig:263-268 -> batchnorm.zig:129-153 (train),
//                            then activateArray (convolutional.zig:268)
//   ref_gpu_conv_bn_backward gradientArray (convolutional.zig:279) -> batchnorm.zig:155-170
//   ref_gpu_sgd_weights      convolutional.zig:332-334
// so the measured time is what the reference spends on the B200 around one convolution.
//
// This library is the per-op GPU baseline and a second parity anchor; the product
// (libdnb200.so) never links or calls it. Each entry returns the cudaError_t of its launch (a
// sequence: of its first failing launch).

#include <cstdint>

#include DNB_REFERENCE_KERNELS

namespace {

constexpr unsigned kBlock = 256;  // darknet_kernels.hip BLOCK, gpu.zig block_size

inline unsigned grid1d(int64_t n) { return (unsigned)((n + kBlock - 1) / kBlock); }

// rolling_momentum (batchnorm.zig:16)
constexpr float kRollingMomentum = 0.99f;

inline int rc() { return (int)cudaGetLastError(); }

// the first failure of a sequence of launches
inline void keep(int &first, int e) {
    if (!first) first = e;
}

}  // namespace

extern "C" {

int ref_gpu_fill(int n, float alpha, float *x, cudaStream_t s) {
    if (n > 0) fill_kernel<<<grid1d(n), kBlock, 0, s>>>(n, alpha, x);
    return rc();
}
int ref_gpu_copy(int n, const float *x, float *y, cudaStream_t s) {
    if (n > 0) copy_kernel<<<grid1d(n), kBlock, 0, s>>>(n, x, y);
    return rc();
}
int ref_gpu_axpy(int n, float alpha, const float *x, float *y, cudaStream_t s) {
    if (n > 0) axpy_kernel<<<grid1d(n), kBlock, 0, s>>>(n, alpha, x, y);
    return rc();
}
int ref_gpu_scal(int n, float alpha, float *x, cudaStream_t s) {
    if (n > 0) scal_kernel<<<grid1d(n), kBlock, 0, s>>>(n, alpha, x);
    return rc();
}
int ref_gpu_activate_array(float *x, int n, int a, cudaStream_t s) {
    if (n > 0) activate_array_kernel<<<grid1d(n), kBlock, 0, s>>>(x, n, a);
    return rc();
}
int ref_gpu_gradient_array(const float *y, int n, int a, float *delta, cudaStream_t s) {
    if (n > 0) gradient_array_kernel<<<grid1d(n), kBlock, 0, s>>>(y, n, a, delta);
    return rc();
}
int ref_gpu_add_bias(float *out, const float *biases, int batch, int filters, int spatial, cudaStream_t s) {
    const int64_t n = (int64_t)batch * filters * spatial;
    if (n > 0) add_bias_kernel<<<grid1d(n), kBlock, 0, s>>>(out, biases, batch, filters, spatial);
    return rc();
}
int ref_gpu_scale_bias(float *out, const float *scales, int batch, int filters, int spatial, cudaStream_t s) {
    const int64_t n = (int64_t)batch * filters * spatial;
    if (n > 0)
        scale_bias_kernel<<<grid1d(n), kBlock, 0, s>>>(out, scales, batch, filters, spatial);
    return rc();
}
// gpu.zig:539-549: spatial == 1 dispatches the per-thread kernel
int ref_gpu_backward_bias(float *bias_updates, const float *delta, int batch, int filters, int spatial,
                          cudaStream_t s) {
    if (filters <= 0) return rc();
    if (spatial == 1)
        backward_bias_conn_kernel<<<grid1d(filters), kBlock, 0, s>>>(bias_updates, delta, batch, filters);
    else
        backward_bias_kernel<<<filters, kBlock, 0, s>>>(bias_updates, delta, batch, filters, spatial);
    return rc();
}
int ref_gpu_backward_scale(const float *x_norm, const float *delta, int batch, int filters, int spatial,
                           float *scale_updates, cudaStream_t s) {
    if (filters > 0)
        backward_scale_kernel<<<filters, kBlock, 0, s>>>(x_norm, delta, batch, filters, spatial, scale_updates);
    return rc();
}
int ref_gpu_mean(const float *x, int batch, int filters, int spatial, float *out, cudaStream_t s) {
    if (filters > 0) fast_mean_kernel<<<filters, kBlock, 0, s>>>(x, batch, filters, spatial, out);
    return rc();
}
int ref_gpu_variance(const float *x, const float *mean, int batch, int filters, int spatial, float *out,
                     cudaStream_t s) {
    if (filters > 0)
        fast_variance_kernel<<<filters, kBlock, 0, s>>>(x, mean, batch, filters, spatial, out);
    return rc();
}
int ref_gpu_normalize(float *x, const float *mean, const float *variance, int batch, int filters, int spatial,
                      cudaStream_t s) {
    const int n = batch * filters * spatial;
    if (n > 0)
        normalize_kernel<<<grid1d(n), kBlock, 0, s>>>(n, x, mean, variance, batch, filters, spatial);
    return rc();
}
int ref_gpu_mean_delta(const float *delta, const float *variance, int batch, int filters, int spatial, float *out,
                       cudaStream_t s) {
    if (filters > 0)
        fast_mean_delta_kernel<<<filters, kBlock, 0, s>>>(delta, variance, batch, filters, spatial, out);
    return rc();
}
int ref_gpu_variance_delta(const float *x, const float *delta, const float *mean, const float *variance, int batch,
                           int filters, int spatial, float *out, cudaStream_t s) {
    if (filters > 0)
        fast_variance_delta_kernel<<<filters, kBlock, 0, s>>>(x, delta, mean, variance, batch, filters, spatial, out);
    return rc();
}
int ref_gpu_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                            const float *variance_delta, int batch, int filters, int spatial, float *delta,
                            cudaStream_t s) {
    const int n = batch * filters * spatial;
    if (n > 0)
        normalize_delta_kernel<<<grid1d(n), kBlock, 0, s>>>(
            n, x, mean, variance,
            mean_delta, variance_delta, batch, filters, spatial, delta);
    return rc();
}

// convolutional.zig:263-268 with batch_normalize, batchnorm.zig:129-153 (state.train):
// `output` holds the convolution's result on entry and the activated layer output on return.
int ref_gpu_conv_bn_forward(float *output, float *x, float *x_norm, float *mean, float *variance,
                            float *rolling_mean, float *rolling_variance, const float *scales, const float *biases,
                            int batch, int filters, int spatial, int act, cudaStream_t s) {
    const int n = batch * filters * spatial;
    int e = 0;
    keep(e, ref_gpu_copy(n, output, x, s));
    keep(e, ref_gpu_mean(output, batch, filters, spatial, mean, s));
    keep(e, ref_gpu_variance(output, mean, batch, filters, spatial, variance, s));
    keep(e, ref_gpu_scal(filters, kRollingMomentum, rolling_mean, s));
    keep(e, ref_gpu_axpy(filters, 1 - kRollingMomentum, mean, rolling_mean, s));
    keep(e, ref_gpu_scal(filters, kRollingMomentum, rolling_variance, s));
    keep(e, ref_gpu_axpy(filters, 1 - kRollingMomentum, variance, rolling_variance, s));
    keep(e, ref_gpu_normalize(output, mean, variance, batch, filters, spatial, s));
    keep(e, ref_gpu_copy(n, output, x_norm, s));
    keep(e, ref_gpu_scale_bias(output, scales, batch, filters, spatial, s));
    keep(e, ref_gpu_add_bias(output, biases, batch, filters, spatial, s));
    keep(e, ref_gpu_activate_array(output, n, act, s));
    return e;
}

// convolutional.zig:279-282, batchnorm.zig:155-170 (state.train): `delta` is dL/d(output)
// on entry and dL/d(conv output) on return; `output` is the forward's activated output.
int ref_gpu_conv_bn_backward(const float *output, float *delta, const float *x, const float *x_norm,
                             const float *mean, const float *variance, const float *scales, float *bias_updates,
                             float *scale_updates, float *mean_delta, float *variance_delta, int batch, int filters,
                             int spatial, int act, cudaStream_t s) {
    const int n = batch * filters * spatial;
    int e = 0;
    keep(e, ref_gpu_gradient_array(output, n, act, delta, s));
    keep(e, ref_gpu_backward_bias(bias_updates, delta, batch, filters, spatial, s));
    keep(e, ref_gpu_backward_scale(x_norm, delta, batch, filters, spatial, scale_updates, s));
    keep(e, ref_gpu_scale_bias(delta, scales, batch, filters, spatial, s));
    keep(e, ref_gpu_mean_delta(delta, variance, batch, filters, spatial, mean_delta, s));
    keep(e, ref_gpu_variance_delta(x, delta, mean, variance, batch, filters, spatial, variance_delta, s));
    keep(e, ref_gpu_normalize_delta(x, mean, variance, mean_delta, variance_delta, batch, filters, spatial, delta, s));
    return e;
}

// convolutional.zig:332-334: the weight part of the SGD update (decay, step, momentum)
int ref_gpu_sgd_weights(int nweights, float learning_rate, float momentum, float decay, int batch, float *weights,
                        float *weight_updates, cudaStream_t s) {
    int e = 0;
    keep(e, ref_gpu_axpy(nweights, -decay * batch, weights, weight_updates, s));
    keep(e, ref_gpu_axpy(nweights, learning_rate / batch, weight_updates, weights, s));
    keep(e, ref_gpu_scal(nweights, momentum, weight_updates, s));
    return e;
}

// launches per call of the sequences above
int ref_gpu_launches_forward(void) { return 12; }
int ref_gpu_launches_backward(void) { return 7; }
int ref_gpu_launches_sgd(void) { return 3; }

}  // extern "C"
