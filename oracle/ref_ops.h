/* TEST INFRASTRUCTURE -- declarations of the CPU oracle (ref_ops.c). */
#ifndef DNB_ORACLE_REF_OPS_H
#define DNB_ORACLE_REF_OPS_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* activations.zig:11-27 (darknet's ACTIVATION numbering) */
enum {
    ACT_LOGISTIC = 0, ACT_RELU = 1, ACT_RELIE = 2, ACT_LINEAR = 3, ACT_RAMP = 4, ACT_TANH = 5, ACT_PLSE = 6,
    ACT_LEAKY = 7, ACT_ELU = 8, ACT_LOGGY = 9, ACT_STAIR = 10, ACT_HARDTAN = 11, ACT_LHTAN = 12, ACT_SELU = 13
};

void oracle_set_threads(int n);
int oracle_get_threads(void);

void ref_fill(float *x, int64_t n, float alpha);
void ref_copy(const float *src, float *dst, int64_t n);
void ref_axpy(float alpha, const float *x, float *y, int64_t n);
void ref_scal(float alpha, float *x, int64_t n);
void ref_mul(const float *x, float *y, int64_t n);
void ref_add_scalar(float alpha, float *x, int64_t n);
void ref_constrain(float alpha, float *x, int64_t n);

float ref_activate(float x, int a);
float ref_gradient(float y, int a);
void ref_activate_array(float *x, int64_t n, int a);
void ref_gradient_array(const float *y, int64_t n, int a, float *delta);

void ref_add_bias(float *out, const float *biases, int64_t batch, int64_t filters, int64_t spatial);
void ref_scale_bias(float *out, const float *scales, int64_t batch, int64_t filters, int64_t spatial);
void ref_backward_bias(float *bias_updates, const float *delta, int64_t batch, int64_t filters, int64_t spatial);
void ref_backward_scale(const float *x_norm, const float *delta, int64_t batch, int64_t filters, int64_t spatial,
                        float *scale_updates);

void ref_mean(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out);
void ref_variance(const float *x, const float *mean, int64_t batch, int64_t filters, int64_t spatial, float *out);
void ref_normalize(float *x, const float *mean, const float *variance, int64_t batch, int64_t filters,
                   int64_t spatial);
void ref_mean_delta(const float *delta, const float *variance, int64_t batch, int64_t filters, int64_t spatial,
                    float *out);
void ref_variance_delta(const float *x, const float *delta, const float *mean, const float *variance, int64_t batch,
                        int64_t filters, int64_t spatial, float *out);
void ref_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                         const float *variance_delta, int64_t batch, int64_t filters, int64_t spatial, float *delta);

void ref_softmax(const float *input, int64_t n, int64_t batch, int64_t batch_offset, int64_t groups,
                 int64_t group_offset, int64_t stride, float temp, float *output);
void ref_softmax_cross_entropy(const float *pred, const float *truth, float *delta, float *err, int64_t n);
float ref_sum_array(const float *a, int64_t n);

void ref_shortcut(int64_t batch, int64_t w1, int64_t h1, int64_t c1, const float *add, int64_t w2, int64_t h2,
                  int64_t c2, float s1, float s2, float *out);

int64_t ref_maxpool_out_dim(int64_t in, int64_t size, int64_t stride, int64_t pad);
void ref_forward_maxpool(int64_t batch, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride, int64_t size,
                         int64_t pad, const float *input, float *output, int32_t *indexes);
void ref_backward_maxpool(int64_t out_n, const float *delta, const int32_t *indexes, float *prev_delta);
void ref_forward_avgpool(int64_t batch, int64_t c, int64_t h, int64_t w, const float *input, float *output);
void ref_backward_avgpool(int64_t batch, int64_t c, int64_t h, int64_t w, const float *out_delta, float *in_delta);

void ref_bn_forward_layer(const float *x, float *y, float *x_saved, float *x_norm, int64_t batch, int64_t filters,
                          int64_t spatial, const float *scales, const float *biases, float *mean, float *variance,
                          float *rolling_mean, float *rolling_variance, int train, int act);
void ref_bn_backward_layer(const float *x, const float *x_norm, const float *y, float *delta, int64_t batch,
                           int64_t filters, int64_t spatial, const float *scales, const float *mean,
                           const float *variance, float *bias_updates, float *scale_updates, float *mean_delta,
                           float *variance_delta, int act);
void ref_sgd_update(float *w, float *wu, int64_t n, float learning_rate, float momentum, float decay, int64_t batch);

#ifdef __cplusplus
}
#endif
#endif
