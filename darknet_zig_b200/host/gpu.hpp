// C++ host mirror of the reference's GPU op layer (src/gpu.zig) over libdnb200.
//
// The reference's host is Zig (0.16); this header keeps its interface for C++ hosts and
// tests: the same `Buf` view (gpu.zig:115-134), the same op names and argument order
// (gpu.zig:483-830), and the same error behaviour -- init-time failures are returned
// to the caller (gpu.zig:41-46, here an exception the caller can handle), a failed launch
// is fatal (std.debug.panic, gpu.zig:443-449, here `Panic`, which callers do not catch in
// normal use). Sizes are size_t as in gpu.zig and widen to int64_t at the ABI (the
// reference narrows them to c_int, gpu.zig:416-418). Every op runs on the legacy default
// stream, as the reference's launches do (cuda.zig:338).
//
// Header-only; link with -ldnb200.
#pragma once

#include <cstddef>
#include <cstdint>
#include <stdexcept>
#include <string>

#include "dnb200.h"

namespace dnb {
namespace gpu {

// The reference's activation codes (activations.zig:11-25).
enum Activation : int {
    logistic = 0, relu = 1, relie = 2, linear = 3, ramp = 4, tanh_ = 5, plse = 6, leaky = 7,
    elu = 8, loggy = 9, stair = 10, hardtan = 11, lhtan = 12, selu = 13
};

// A failed op: the reference panics here (gpu.zig:443-449).
struct Panic : std::runtime_error {
    int status;
    Panic(const char *what, int s)
        : std::runtime_error(std::string(what) + ": " + dnb_error_string(s) + ": " + dnb_last_error_detail()),
          status(s) {}
};
// A failed initialisation: the reference returns an error (gpu.zig:41-46).
struct InitError : std::runtime_error {
    int status;
    InitError(const char *what, int s)
        : std::runtime_error(std::string(what) + ": " + dnb_error_string(s) + ": " + dnb_last_error_detail()),
          status(s) {}
};

inline void check(const char *what, dnb_status s) {
    if (s != DNB_OK) throw Panic(what, s);
}

// gpu.zig:115-134: a non-owning view of device floats.
struct Buf {
    void *ptr = nullptr;
    size_t len = 0;  // in floats
    bool isNull() const { return ptr == nullptr; }
    // n floats in: the reference's pointer arithmetic on float* (gpu.zig:128-133)
    Buf offset(size_t n) const {
        if (!ptr) return {};
        return {static_cast<char *>(ptr) + n * sizeof(float), len - n};
    }
    float *f() const { return static_cast<float *>(ptr); }
    int32_t *i() const { return static_cast<int32_t *>(ptr); }
};

inline int64_t i64(size_t v) { return static_cast<int64_t>(v); }

// ---- device and memory: gpu.zig:259-410 ------------------------------------------------

inline void init(int device) {
    const dnb_status s = dnb_init(device);
    if (s != DNB_OK) throw InitError("gpu.init", s);
}
inline int deviceCount() {
    int n = 0;
    const dnb_status s = dnb_device_count(&n);
    if (s != DNB_OK) throw InitError("gpu.deviceCount", s);
    return n;
}
// gpu.alloc: zero-filled (gpu.zig:362-369)
inline Buf alloc(size_t n) {
    void *p = nullptr;
    check("gpu.alloc", dnb_malloc(&p, n * sizeof(float)));
    return {p, n};
}
inline void free(Buf b) {
    if (b.ptr) check("gpu.free", dnb_free(b.ptr));
}
inline void push(Buf dst, const float *src, size_t n) {
    check("gpu.push", dnb_push(dst.ptr, src, n * sizeof(float), nullptr));
    check("gpu.push", dnb_stream_sync(nullptr));
}
inline void pull(Buf src, float *dst, size_t n) {
    check("gpu.pull", dnb_pull(dst, src.ptr, n * sizeof(float), nullptr));
    check("gpu.pull", dnb_stream_sync(nullptr));
}
// gpu.make: allocate and upload (gputest.zig's helper)
inline Buf make(const float *host, size_t n) {
    Buf b = alloc(n);
    push(b, host, n);
    return b;
}
inline void sync() { check("gpu.sync", dnb_sync()); }
inline void setSyncAfterLaunch(bool on) { check("gpu.setSyncAfterLaunch", dnb_set_sync_after_launch(on ? 1 : 0)); }

// ---- elementwise: gpu.zig:483-518 ------------------------------------------------------

inline void fill(Buf x, size_t n, float alpha) { check("gpu.fill", dnb_fill(x.f(), i64(n), alpha, nullptr)); }
inline void copy(size_t n, Buf x, Buf y) { check("gpu.copy", dnb_copy(i64(n), x.f(), y.f(), nullptr)); }
inline void axpy(size_t n, float alpha, Buf x, Buf y) {
    check("gpu.axpy", dnb_axpy(i64(n), alpha, x.f(), y.f(), nullptr));
}
inline void scal(size_t n, float alpha, Buf x) { check("gpu.scal", dnb_scal(i64(n), alpha, x.f(), nullptr)); }
inline void mul(size_t n, Buf x, Buf y) { check("gpu.mul", dnb_mul(i64(n), x.f(), y.f(), nullptr)); }
inline void addScalar(size_t n, float alpha, Buf x) {
    check("gpu.addScalar", dnb_add_scalar(i64(n), alpha, x.f(), nullptr));
}
inline void constrain(size_t n, float alpha, Buf x) {
    check("gpu.constrain", dnb_constrain(i64(n), alpha, x.f(), nullptr));
}
inline void activateArray(Buf x, size_t n, int a) {
    check("gpu.activateArray", dnb_activate_array(x.f(), i64(n), a, nullptr));
}
inline void gradientArray(Buf x, size_t n, int a, Buf delta) {
    check("gpu.gradientArray", dnb_gradient_array(x.f(), i64(n), a, delta.f(), nullptr));
}

// ---- bias, scale, batchnorm pieces: gpu.zig:520-613 ------------------------------------

inline void addBias(Buf output, Buf biases, size_t batch, size_t filters, size_t spatial) {
    check("gpu.addBias", dnb_add_bias(output.f(), biases.f(), i64(batch), i64(filters), i64(spatial), nullptr));
}
inline void scaleBias(Buf output, Buf scales, size_t batch, size_t filters, size_t spatial) {
    check("gpu.scaleBias", dnb_scale_bias(output.f(), scales.f(), i64(batch), i64(filters), i64(spatial), nullptr));
}
inline void backwardBias(Buf bias_updates, Buf delta, size_t batch, size_t filters, size_t spatial) {
    check("gpu.backwardBias",
          dnb_backward_bias(bias_updates.f(), delta.f(), i64(batch), i64(filters), i64(spatial), nullptr));
}
inline void backwardScale(Buf x_norm, Buf delta, size_t batch, size_t filters, size_t spatial, Buf scale_updates) {
    check("gpu.backwardScale", dnb_backward_scale(x_norm.f(), delta.f(), i64(batch), i64(filters), i64(spatial),
                                                  scale_updates.f(), nullptr));
}
inline void mean(Buf x, size_t batch, size_t filters, size_t spatial, Buf out) {
    check("gpu.mean", dnb_mean(x.f(), i64(batch), i64(filters), i64(spatial), out.f(), nullptr));
}
inline void variance(Buf x, Buf mean_in, size_t batch, size_t filters, size_t spatial, Buf out) {
    check("gpu.variance", dnb_variance(x.f(), mean_in.f(), i64(batch), i64(filters), i64(spatial), out.f(), nullptr));
}
inline void normalize(Buf x, Buf mean_in, Buf variance_in, size_t batch, size_t filters, size_t spatial) {
    check("gpu.normalize",
          dnb_normalize(x.f(), mean_in.f(), variance_in.f(), i64(batch), i64(filters), i64(spatial), nullptr));
}
inline void meanDelta(Buf delta, Buf variance_in, size_t batch, size_t filters, size_t spatial, Buf out) {
    check("gpu.meanDelta",
          dnb_mean_delta(delta.f(), variance_in.f(), i64(batch), i64(filters), i64(spatial), out.f(), nullptr));
}
inline void varianceDelta(Buf x, Buf delta, Buf mean_in, Buf variance_in, size_t batch, size_t filters,
                          size_t spatial, Buf out) {
    check("gpu.varianceDelta", dnb_variance_delta(x.f(), delta.f(), mean_in.f(), variance_in.f(), i64(batch),
                                                  i64(filters), i64(spatial), out.f(), nullptr));
}
inline void normalizeDelta(Buf x, Buf mean_in, Buf variance_in, Buf mean_delta, Buf variance_delta, size_t batch,
                           size_t filters, size_t spatial, Buf delta) {
    check("gpu.normalizeDelta",
          dnb_normalize_delta(x.f(), mean_in.f(), variance_in.f(), mean_delta.f(), variance_delta.f(), i64(batch),
                              i64(filters), i64(spatial), delta.f(), nullptr));
}

// ---- softmax, pooling, shortcut: gpu.zig:615-802 ---------------------------------------

inline void softmax(Buf input, size_t n, size_t batch, size_t batch_offset, size_t groups, size_t group_offset,
                    size_t stride, float temp, Buf output) {
    check("gpu.softmax", dnb_softmax(input.f(), i64(n), i64(batch), i64(batch_offset), i64(groups),
                                     i64(group_offset), i64(stride), temp, output.f(), nullptr));
}
inline void softmaxCrossEntropy(size_t n, Buf pred, Buf truth, Buf delta, Buf err) {
    check("gpu.softmaxCrossEntropy",
          dnb_softmax_cross_entropy(i64(n), pred.f(), truth.f(), delta.f(), err.f(), nullptr));
}
// indexes: int32 in a float-sized buffer (gpu.zig:371-375)
inline void forwardMaxpool(size_t out_n, size_t in_h, size_t in_w, size_t in_c, size_t stride, size_t size,
                           size_t pad, Buf input, Buf output, Buf indexes) {
    check("gpu.forwardMaxpool", dnb_forward_maxpool(i64(out_n), i64(in_h), i64(in_w), i64(in_c), i64(stride),
                                                    i64(size), i64(pad), input.f(), output.f(), indexes.i(),
                                                    nullptr));
}
inline void backwardMaxpool(size_t in_n, size_t in_h, size_t in_w, size_t in_c, size_t stride, size_t size,
                            size_t pad, Buf delta, Buf prev_delta, Buf indexes) {
    check("gpu.backwardMaxpool", dnb_backward_maxpool(i64(in_n), i64(in_h), i64(in_w), i64(in_c), i64(stride),
                                                      i64(size), i64(pad), delta.f(), prev_delta.f(), indexes.i(),
                                                      nullptr));
}
inline void forwardAvgpool(size_t n, size_t w, size_t h, size_t c, Buf input, Buf output) {
    check("gpu.forwardAvgpool", dnb_forward_avgpool(i64(n), i64(w), i64(h), i64(c), input.f(), output.f(), nullptr));
}
inline void backwardAvgpool(size_t n, size_t w, size_t h, size_t c, Buf in_delta, Buf out_delta) {
    check("gpu.backwardAvgpool",
          dnb_backward_avgpool(i64(n), i64(w), i64(h), i64(c), in_delta.f(), out_delta.f(), nullptr));
}
inline void shortcut(size_t batch, size_t w1, size_t h1, size_t c1, Buf add, size_t w2, size_t h2, size_t c2,
                     float s1, float s2, Buf out) {
    check("gpu.shortcut", dnb_shortcut(i64(batch), i64(w1), i64(h1), i64(c1), add.f(), i64(w2), i64(h2), i64(c2), s1,
                                       s2, out.f(), nullptr));
}

// ---- fused entries (one kernel where the reference issues a sequence) -----------------

// batchnorm.forwardGpu train branch + activate (batchnorm.zig:129-152, convolutional.zig:269)
inline void bnActForwardTrain(Buf x, Buf y, Buf x_norm, size_t batch, size_t filters, size_t spatial, Buf scales,
                              Buf biases, Buf mean_out, Buf variance_out, Buf rolling_mean, Buf rolling_variance,
                              int act) {
    check("gpu.bnActForwardTrain",
          dnb_bn_act_forward_train(x.f(), y.f(), x_norm.f(), i64(batch), i64(filters), i64(spatial), scales.f(),
                                   biases.f(), mean_out.f(), variance_out.f(), rolling_mean.f(),
                                   rolling_variance.f(), act, nullptr));
}
inline void bnActForwardInfer(Buf x, Buf y, size_t batch, size_t filters, size_t spatial, Buf scales, Buf biases,
                              Buf rolling_mean, Buf rolling_variance, int act) {
    check("gpu.bnActForwardInfer",
          dnb_bn_act_forward_infer(x.f(), y.f(), i64(batch), i64(filters), i64(spatial), scales.f(), biases.f(),
                                   rolling_mean.f(), rolling_variance.f(), act, nullptr));
}
// gradientArray + batchnorm.backwardGpu (convolutional.zig:280, batchnorm.zig:155-169)
inline void bnActBackward(Buf x, Buf y, Buf delta, Buf dx, size_t batch, size_t filters, size_t spatial, Buf scales,
                          Buf biases, Buf mean_in, Buf variance_in, Buf bias_updates, Buf scale_updates,
                          Buf mean_delta, Buf variance_delta, int act) {
    check("gpu.bnActBackward",
          dnb_bn_act_backward(x.f(), y.f(), delta.f(), dx.f(), i64(batch), i64(filters), i64(spatial), scales.f(),
                              biases.f(), mean_in.f(), variance_in.f(), bias_updates.f(), scale_updates.f(),
                              mean_delta.f(), variance_delta.f(), act, nullptr));
}
// convolutional.updateGpu's weight update (convolutional.zig:332-334)
inline void sgdMomentum(size_t n, Buf weights, Buf weight_updates, float learning_rate, float momentum, float decay,
                        size_t batch) {
    check("gpu.sgdMomentum", dnb_sgd_momentum(i64(n), weights.f(), weight_updates.f(), learning_rate, momentum, decay,
                                              i64(batch), nullptr));
}
// misc.forwardSoftmaxGpu (misc.zig:59-72); cost may be a null Buf
inline void softmaxXent(Buf input, Buf truth, size_t n, size_t batch, float temp, Buf output, Buf delta, Buf err,
                        Buf cost) {
    check("gpu.softmaxXent", dnb_softmax_xent(input.f(), truth.f(), i64(n), i64(batch), temp, output.f(), delta.f(),
                                              err.f(), cost.f(), nullptr));
}

}  // namespace gpu
}  // namespace dnb
