// TEST INFRASTRUCTURE -- the reference's own device kernels, run on the host.
//
// The reference kernel file (src/kernels/darknet_kernels.hip, path passed in as
// DNB_REFERENCE_KERNELS at build time) is #included unchanged and compiled by g++
// through hip_host_shim.h. Each ref_emu_* entry point launches one of those kernels with
// the grid the reference's dispatcher uses (src/gpu.zig:420-477): launch1d =
// ceil(n/256) blocks of 256 threads, launchPerFilter = one 256-thread block per filter.
//
// Built with -ffp-contract=fast (the build passes -ffp-contract=off first and this file
// re-enables contraction below) so that a*b+c is fused the way nvcc fuses it by default.
//
// This library exists to pin the C restatement (ref_ops.c) against code that is the
// reference's own: tests compare the two on the reference's gputest shapes.
#pragma GCC optimize("fp-contract=fast")

#include <cstdint>
#include <thread>
#include <vector>

#include "hip_host_shim.h"

thread_local dnb_dim3 dnb_thread_idx;
thread_local dnb_dim3 dnb_block_idx;
dnb_dim3 dnb_block_dim;
dnb_dim3 dnb_grid_dim;
std::barrier<> *dnb_block_barrier = nullptr;

#include DNB_REFERENCE_KERNELS

namespace {

constexpr unsigned kBlock = 256;  // darknet_kernels.hip:35, gpu.zig:58

template <class Body>
void run_grid(unsigned grid, unsigned block, bool uses_barrier, Body body) {
    dnb_grid_dim = {grid, 1, 1};
    dnb_block_dim = {block, 1, 1};
    for (unsigned b = 0; b < grid; ++b) {
        if (!uses_barrier) {
            dnb_block_idx = {b, 0, 0};
            for (unsigned t = 0; t < block; ++t) {
                dnb_thread_idx = {t, 0, 0};
                body();
            }
            continue;
        }
        std::barrier<> bar(block);
        dnb_block_barrier = &bar;
        std::vector<std::thread> threads;
        threads.reserve(block);
        for (unsigned t = 0; t < block; ++t) {
            threads.emplace_back([b, t, &body] {
                dnb_block_idx = {b, 0, 0};
                dnb_thread_idx = {t, 0, 0};
                body();
            });
        }
        for (auto &th : threads) th.join();
        dnb_block_barrier = nullptr;
    }
}

unsigned grid1d(int64_t n) { return (unsigned)((n + kBlock - 1) / kBlock); }

}  // namespace

extern "C" {

void ref_emu_activate_array(float *x, int n, int a) {
    run_grid(grid1d(n), kBlock, false, [&] { activate_array_kernel(x, n, a); });
}
void ref_emu_gradient_array(const float *y, int n, int a, float *delta) {
    run_grid(grid1d(n), kBlock, false, [&] { gradient_array_kernel(y, n, a, delta); });
}
void ref_emu_fill(int n, float alpha, float *x) {
    run_grid(grid1d(n), kBlock, false, [&] { fill_kernel(n, alpha, x); });
}
void ref_emu_copy(int n, const float *x, float *y) {
    run_grid(grid1d(n), kBlock, false, [&] { copy_kernel(n, x, y); });
}
void ref_emu_axpy(int n, float alpha, const float *x, float *y) {
    run_grid(grid1d(n), kBlock, false, [&] { axpy_kernel(n, alpha, x, y); });
}
void ref_emu_scal(int n, float alpha, float *x) {
    run_grid(grid1d(n), kBlock, false, [&] { scal_kernel(n, alpha, x); });
}
void ref_emu_mul(int n, const float *x, float *y) {
    run_grid(grid1d(n), kBlock, false, [&] { mul_kernel(n, x, y); });
}
void ref_emu_add_scalar(int n, float alpha, float *x) {
    run_grid(grid1d(n), kBlock, false, [&] { add_scalar_kernel(n, alpha, x); });
}
void ref_emu_constrain(int n, float alpha, float *x) {
    run_grid(grid1d(n), kBlock, false, [&] { constrain_kernel(n, alpha, x); });
}
void ref_emu_add_bias(float *out, const float *biases, int batch, int filters, int spatial) {
    run_grid(grid1d((int64_t)batch * filters * spatial), kBlock, false,
             [&] { add_bias_kernel(out, biases, batch, filters, spatial); });
}
void ref_emu_scale_bias(float *out, const float *scales, int batch, int filters, int spatial) {
    run_grid(grid1d((int64_t)batch * filters * spatial), kBlock, false,
             [&] { scale_bias_kernel(out, scales, batch, filters, spatial); });
}
// gpu.zig:528-540: spatial == 1 dispatches the per-thread kernel
void ref_emu_backward_bias(float *bias_updates, const float *delta, int batch, int filters, int spatial) {
    if (spatial == 1) {
        run_grid(grid1d(filters), kBlock, false,
                 [&] { backward_bias_conn_kernel(bias_updates, delta, batch, filters); });
    } else {
        run_grid(filters, kBlock, true, [&] { backward_bias_kernel(bias_updates, delta, batch, filters, spatial); });
    }
}
void ref_emu_backward_scale(const float *x_norm, const float *delta, int batch, int filters, int spatial,
                            float *scale_updates) {
    run_grid(filters, kBlock, true,
             [&] { backward_scale_kernel(x_norm, delta, batch, filters, spatial, scale_updates); });
}
void ref_emu_mean(const float *x, int batch, int filters, int spatial, float *out) {
    run_grid(filters, kBlock, true, [&] { fast_mean_kernel(x, batch, filters, spatial, out); });
}
void ref_emu_variance(const float *x, const float *mean, int batch, int filters, int spatial, float *out) {
    run_grid(filters, kBlock, true, [&] { fast_variance_kernel(x, mean, batch, filters, spatial, out); });
}
void ref_emu_normalize(float *x, const float *mean, const float *variance, int batch, int filters, int spatial) {
    const int n = batch * filters * spatial;
    run_grid(grid1d(n), kBlock, false,
             [&] { normalize_kernel(n, x, mean, variance, batch, filters, spatial); });
}
void ref_emu_mean_delta(const float *delta, const float *variance, int batch, int filters, int spatial, float *out) {
    run_grid(filters, kBlock, true, [&] { fast_mean_delta_kernel(delta, variance, batch, filters, spatial, out); });
}
void ref_emu_variance_delta(const float *x, const float *delta, const float *mean, const float *variance, int batch,
                            int filters, int spatial, float *out) {
    run_grid(filters, kBlock, true,
             [&] { fast_variance_delta_kernel(x, delta, mean, variance, batch, filters, spatial, out); });
}
void ref_emu_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                             const float *variance_delta, int batch, int filters, int spatial, float *delta) {
    const int n = batch * filters * spatial;
    run_grid(grid1d(n), kBlock, false, [&] {
        normalize_delta_kernel(n, x, mean, variance, mean_delta, variance_delta, batch, filters, spatial, delta);
    });
}
void ref_emu_softmax(const float *input, int n, int batch, int batch_offset, int groups, int group_offset, int stride,
                     float temp, float *output) {
    run_grid(grid1d((int64_t)batch * groups), kBlock, false, [&] {
        softmax_kernel(input, n, batch, batch_offset, groups, group_offset, stride, temp, output);
    });
}
void ref_emu_softmax_x_ent(int n, const float *pred, const float *truth, float *delta, float *err) {
    run_grid(grid1d(n), kBlock, false, [&] { softmax_x_ent_kernel(n, pred, truth, delta, err); });
}
void ref_emu_forward_maxpool(int out_n, int in_h, int in_w, int in_c, int stride, int size, int pad,
                             const float *input, float *output, int *indexes) {
    run_grid(grid1d(out_n), kBlock, false, [&] {
        forward_maxpool_kernel(out_n, in_h, in_w, in_c, stride, size, pad, input, output, indexes);
    });
}
void ref_emu_backward_maxpool(int in_n, int in_h, int in_w, int in_c, int stride, int size, int pad,
                              const float *delta, float *prev_delta, const int *indexes) {
    run_grid(grid1d(in_n), kBlock, false, [&] {
        backward_maxpool_kernel(in_n, in_h, in_w, in_c, stride, size, pad, delta, prev_delta, indexes);
    });
}
void ref_emu_forward_avgpool(int n, int w, int h, int c, const float *input, float *output) {
    run_grid(grid1d(n), kBlock, false, [&] { forward_avgpool_kernel(n, w, h, c, input, output); });
}
void ref_emu_backward_avgpool(int n, int w, int h, int c, float *in_delta, const float *out_delta) {
    run_grid(grid1d(n), kBlock, false, [&] { backward_avgpool_kernel(n, w, h, c, in_delta, out_delta); });
}
// gpu.zig:762-790 computes the resampling parameters on the host before the launch
void ref_emu_shortcut(int batch, int w1, int h1, int c1, const float *add, int w2, int h2, int c2, float s1, float s2,
                      float *out) {
    int stride = w1 / w2, sample = w2 / w1;
    if (stride < 1) stride = 1;
    if (sample < 1) sample = 1;
    const int minw = w1 < w2 ? w1 : w2, minh = h1 < h2 ? h1 : h2, minc = c1 < c2 ? c1 : c2;
    const int size = batch * minw * minh * minc;
    run_grid(grid1d(size), kBlock, false, [&] {
        shortcut_kernel(size, minw, minh, minc, stride, sample, batch, w1, h1, c1, add, w2, h2, c2, s1, s2, out);
    });
}

}  // extern "C"
