/*
 * dnb200.h -- C ABI of libdnb200.so, the sm_100a (B200) implementation of darknet-zig's
 * elementwise, reduction and broadcast tensor ops.
 *
 * This ABI replaces the reference's vendor shim (src/cuda/cuda.zig) and the GPU half of
 * its array-op layer (src/gpu.zig). Each entry below names the reference function it
 * stands in for. Conventions, all inherited from the reference:
 *   - tensors are NCHW fp32, index = ((b*C + c)*H + y)*W + x, spatial = H*W
 *     (src/blas.zig:51, src/kernels/darknet_kernels.hip:14-18);
 *   - `delta` is dL/d(output) and is accumulated into where the reference accumulates;
 *   - activation gradients take the activation OUTPUT y (src/activations.zig:1-7);
 *   - activation codes are darknet's ACTIVATION numbering (src/activations.zig:11-27);
 *   - maxpool indices are int32 flat input indices (src/layers/pooling.zig:42,79).
 * Differences from the reference ABI:
 *   - sizes are int64_t (the reference passes c_int, src/gpu.zig:416-418);
 *   - every op takes a stream (NULL = the legacy default stream the reference uses,
 *     src/cuda/cuda.zig:338) and returns a dnb_status instead of panicking
 *     (src/gpu.zig:48-55,443-449);
 *   - pointers are raw device pointers owned by the caller (Buf{ptr,len} without the
 *     length, src/gpu.zig:117-134). The library owns only its per-stream workspace
 *     (per-channel partials, the fused kernels' tagged records and launch epoch) and the
 *     comm state.
 * Threading: calls on one stream must come from one host thread at a time.
 */
#ifndef DNB200_H
#define DNB200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int dnb_status;
typedef void *dnb_stream; /* a cudaStream_t / CUstream; NULL = legacy default stream */
typedef void *dnb_comm;   /* a sync-BN communicator (dnb_comm_init); NULL = none */
typedef void *dnb_dpsgd;  /* a data-parallel weight-update group (dnb_dpsgd_init) */

enum {
    DNB_OK = 0,
    DNB_ERR_INVALID = 1,     /* bad argument (size, alignment, null pointer) */
    DNB_ERR_CUDA = 2,        /* a CUDA runtime call failed; dnb_last_error_detail() says which */
    DNB_ERR_TIMEOUT = 3,     /* a bounded device-side wait gave up; the op's outputs are undefined */
    DNB_ERR_NOT_INIT = 4,    /* dnb_init() was not called on this thread's device */
    DNB_ERR_UNSUPPORTED = 5, /* shape or option outside what the kernels implement */
    DNB_ERR_COMM = 6,        /* sync-BN communicator error */
    DNB_ERR_NO_MEMORY = 7
};

/* activations.zig:11-27 */
enum {
    DNB_ACT_LOGISTIC = 0, DNB_ACT_RELU = 1, DNB_ACT_RELIE = 2, DNB_ACT_LINEAR = 3, DNB_ACT_RAMP = 4,
    DNB_ACT_TANH = 5, DNB_ACT_PLSE = 6, DNB_ACT_LEAKY = 7, DNB_ACT_ELU = 8, DNB_ACT_LOGGY = 9,
    DNB_ACT_STAIR = 10, DNB_ACT_HARDTAN = 11, DNB_ACT_LHTAN = 12, DNB_ACT_SELU = 13
};

/* ------------------------------------------------------------------------------------ */
/* device and memory -- replaces the vendor shim contract of src/gpu.zig:4-11           */
/* (CUDA implementation src/cuda/cuda.zig:248-339) and gpu.zig:362-410                  */
/* ------------------------------------------------------------------------------------ */

/* errorString, cuda.zig:135-172 */
const char *dnb_error_string(dnb_status s);
/* the most recent failure on this host thread, with the CUDA call that caused it */
const char *dnb_last_error_detail(void);
/* initPlatform + setDevice, cuda.zig:248-271 / gpu.zig:259-347. Makes `device` current on
 * the calling thread and sets up its per-device state. */
dnb_status dnb_init(int device);
/* deviceCount, cuda.zig:254-259 */
dnb_status dnb_device_count(int *count);
/* deviceName, cuda.zig:273-277 */
dnb_status dnb_device_name(int device, char *buf, int len);
/* memInfo, cuda.zig:279-281 */
dnb_status dnb_mem_info(size_t *free_bytes, size_t *total_bytes);
/* gpu.alloc, gpu.zig:362-369: zero-filled device allocation */
dnb_status dnb_malloc(void **ptr, size_t bytes);
/* gpu.free, gpu.zig:384-387, cuda.zig:295-297 */
dnb_status dnb_free(void *ptr);
/* memsetZero, cuda.zig:299-301 (async on `stream`) */
dnb_status dnb_memset_zero(void *ptr, size_t bytes, dnb_stream stream);
/* gpu.push / copyToDevice, gpu.zig:389-393, cuda.zig:303-305 (async on `stream`) */
dnb_status dnb_push(void *dst_device, const void *src_host, size_t bytes, dnb_stream stream);
/* gpu.pull / copyToHost, gpu.zig:395-405, cuda.zig:307-309 (async on `stream`) */
dnb_status dnb_pull(void *dst_host, const void *src_device, size_t bytes, dnb_stream stream);
/* gpu.sync / synchronize, gpu.zig:407-410, cuda.zig:311-313 */
dnb_status dnb_sync(void);
dnb_status dnb_stream_sync(dnb_stream stream);
/* setSyncAfterLaunch / DARKNET_GPU_SYNC, gpu.zig:173-183,451-464 (gpu.zig:181): when on, every op
 * synchronises its stream and reports a fault against the op that caused it. */
dnb_status dnb_set_sync_after_launch(int on);
/* Reads and clears the device-side error word of this device (set by a bounded wait that
 * gave up). Synchronises the device. Returns DNB_ERR_TIMEOUT if a wait had expired. */
dnb_status dnb_check_device_error(void);
/* Number of device-side launches (kernels and memsets) this library has issued in this
 * process, all devices and threads together. No counterpart in the reference; it lets a
 * caller check how many launches an op costs. */
dnb_status dnb_launch_count(unsigned long long *count);
/* Sets how long a device-side wait may spin before it gives up (default 2000 ms). */
dnb_status dnb_set_wait_limit_ms(int ms);

/* ------------------------------------------------------------------------------------ */
/* elementwise BLAS -- gpu.zig:483-518, blas.zig:13-46                                   */
/* ------------------------------------------------------------------------------------ */

/* gpu.fill, gpu.zig:483-485 / blas.fill blas.zig:13-15 */
dnb_status dnb_fill(float *x, int64_t n, float alpha, dnb_stream stream);
/* gpu.copy, gpu.zig:487-489 / blas.copy blas.zig:17-19 */
dnb_status dnb_copy(int64_t n, const float *x, float *y, dnb_stream stream);
/* gpu.axpy, gpu.zig:491-493 / blas.axpy blas.zig:21-24: y += alpha*x, one fused rounding */
dnb_status dnb_axpy(int64_t n, float alpha, const float *x, float *y, dnb_stream stream);
/* gpu.scal, gpu.zig:495-497 / blas.scal blas.zig:26-29 */
dnb_status dnb_scal(int64_t n, float alpha, float *x, dnb_stream stream);
/* gpu.mul, gpu.zig:499-501 / blas.mul blas.zig:31-33: y *= x */
dnb_status dnb_mul(int64_t n, const float *x, float *y, dnb_stream stream);
/* gpu.addScalar, gpu.zig:503-505 (add_scalar_kernel, darknet_kernels.hip:150-153) */
dnb_status dnb_add_scalar(int64_t n, float alpha, float *x, dnb_stream stream);
/* gpu.constrainArray, gpu.zig:507-509 / blas.constrainArray blas.zig:44-46 */
dnb_status dnb_constrain(int64_t n, float alpha, float *x, dnb_stream stream);
/* gpu.activateArray, gpu.zig:515-517 / activations.activateArray activations.zig:107-125 */
dnb_status dnb_activate_array(float *x, int64_t n, int act, dnb_stream stream);
/* gpu.gradientArray, gpu.zig:519-521 / activations.gradientArray activations.zig:127-143 */
dnb_status dnb_gradient_array(const float *y, int64_t n, int act, float *delta, dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* bias / scale -- gpu.zig:527-555, blas.zig:53-100                                      */
/* ------------------------------------------------------------------------------------ */

/* gpu.addBias, gpu.zig:527-531 / blas.addBias blas.zig:53-61 */
dnb_status dnb_add_bias(float *output, const float *biases, int64_t batch, int64_t filters, int64_t spatial,
                        dnb_stream stream);
/* gpu.scaleBias, gpu.zig:533-537 / blas.scaleBias blas.zig:63-71 */
dnb_status dnb_scale_bias(float *output, const float *scales, int64_t batch, int64_t filters, int64_t spatial,
                          dnb_stream stream);
/* gpu.backwardBias, gpu.zig:539-549 / blas.backwardBias blas.zig:73-82: bias_updates += sum */
dnb_status dnb_backward_bias(float *bias_updates, const float *delta, int64_t batch, int64_t filters,
                             int64_t spatial, dnb_stream stream);
/* gpu.backwardScale, gpu.zig:551-555 / blas.backwardScale blas.zig:84-100 */
dnb_status dnb_backward_scale(const float *x_norm, const float *delta, int64_t batch, int64_t filters,
                              int64_t spatial, float *scale_updates, dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* batch normalisation pieces -- gpu.zig:561-612, blas.zig:106-204                        */
/* ------------------------------------------------------------------------------------ */

/* gpu.mean, gpu.zig:561-565 / blas.mean blas.zig:106-116 */
dnb_status dnb_mean(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out,
                    dnb_stream stream);
/* gpu.variance, gpu.zig:567-571 / blas.variance blas.zig:121-135 (unbiased) */
dnb_status dnb_variance(const float *x, const float *mean, int64_t batch, int64_t filters, int64_t spatial,
                        float *out, dnb_stream stream);
/* gpu.normalize, gpu.zig:573-578 / blas.normalize blas.zig:137-146 (x*1/(sqrt(v)+1e-6)) */
dnb_status dnb_normalize(float *x, const float *mean, const float *variance, int64_t batch, int64_t filters,
                         int64_t spatial, dnb_stream stream);
/* gpu.meanDelta, gpu.zig:580-584 / blas.meanDelta blas.zig:148-157 */
dnb_status dnb_mean_delta(const float *delta, const float *variance, int64_t batch, int64_t filters,
                          int64_t spatial, float *out, dnb_stream stream);
/* gpu.varianceDelta, gpu.zig:586-590 / blas.varianceDelta blas.zig:159-178 */
dnb_status dnb_variance_delta(const float *x, const float *delta, const float *mean, const float *variance,
                              int64_t batch, int64_t filters, int64_t spatial, float *out, dnb_stream stream);
/* gpu.normalizeDelta, gpu.zig:592-612 / blas.normalizeDelta blas.zig:180-204 */
dnb_status dnb_normalize_delta(const float *x, const float *mean, const float *variance, const float *mean_delta,
                               const float *variance_delta, int64_t batch, int64_t filters, int64_t spatial,
                               float *delta, dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* softmax and losses -- gpu.zig:614-633, blas.zig:213-252, misc.zig:41-77                */
/* ------------------------------------------------------------------------------------ */

/* gpu.softmax, gpu.zig:614-629 / blas.softmax blas.zig:225-242 */
dnb_status dnb_softmax(const float *input, int64_t n, int64_t batch, int64_t batch_offset, int64_t groups,
                       int64_t group_offset, int64_t stride, float temp, float *output, dnb_stream stream);
/* gpu.softmaxCrossEntropy, gpu.zig:631-633 / blas.softmaxCrossEntropy blas.zig:247-252 */
dnb_status dnb_softmax_cross_entropy(int64_t n, const float *pred, const float *truth, float *delta, float *err,
                                     dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* pooling and shortcut -- gpu.zig:725-802, pooling.zig, blas.zig:290-322                  */
/* ------------------------------------------------------------------------------------ */

/* gpu.forwardMaxpool, gpu.zig:725-741 / pooling.forwardMaxpool pooling.zig:59-93.
 * out_n = batch*in_c*out_h*out_w; out = (in + pad - size)/stride + 1 (pooling.zig:33-34). */
dnb_status dnb_forward_maxpool(int64_t out_n, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride,
                               int64_t size, int64_t pad, const float *input, float *output, int32_t *indexes,
                               dnb_stream stream);
/* gpu.backwardMaxpool, gpu.zig:743-759 / pooling.backwardMaxpool pooling.zig:95-103:
 * prev_delta[indexes[i]] += delta[i], contributions added in increasing i. in_n = batch*in_c*in_h*in_w. */
dnb_status dnb_backward_maxpool(int64_t in_n, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride,
                                int64_t size, int64_t pad, const float *delta, float *prev_delta,
                                const int32_t *indexes, dnb_stream stream);
/* gpu.forwardAvgpool, gpu.zig:761-763 / pooling.forwardAvgpool pooling.zig:146-158 (n = batch*c) */
dnb_status dnb_forward_avgpool(int64_t n, int64_t w, int64_t h, int64_t c, const float *input, float *output,
                               dnb_stream stream);
/* gpu.backwardAvgpool, gpu.zig:765-767 / pooling.backwardAvgpool pooling.zig:160-172 */
dnb_status dnb_backward_avgpool(int64_t n, int64_t w, int64_t h, int64_t c, float *in_delta,
                                const float *out_delta, dnb_stream stream);
/* gpu.shortcut, gpu.zig:773-802 / blas.shortcut blas.zig:290-322: out = s1*out + s2*add */
dnb_status dnb_shortcut(int64_t batch, int64_t w1, int64_t h1, int64_t c1, const float *add, int64_t w2,
                        int64_t h2, int64_t c2, float s1, float s2, float *out, dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* fused entries -- one kernel where the reference issues a sequence                     */
/* ------------------------------------------------------------------------------------ */

/* Batchnorm training forward + activation in one HBM pass: replaces
 * batchnorm.forwardGpu (batchnorm.zig:129-153, train branch) followed by
 * gpu.activateArray (convolutional.zig:269).
 *   x       [batch,filters,spatial] conv output; read only. It plays the role of the
 *           reference's l.x (the saved pre-BN copy, batchnorm.zig:134) for the backward.
 *   y       activated output (l.output); may alias x.
 *   x_norm  optional (NULL = not written): the normalised x (l.x_norm, batchnorm.zig:146).
 *   mean, variance  out: batch statistics (unbiased variance, blas.zig:118-135).
 *   rolling_mean, rolling_variance  in/out: r = r*0.99 then r += 0.01*stat with one fused
 *           rounding (scal + axpy, batchnorm.zig:140-143).
 * Per element: y = act(((x - mean) * (1/(sqrt(var)+1e-6))) * scale + bias), in that order
 * and without fused rounding, as normalize + scaleBias + addBias + activate. */
dnb_status dnb_bn_act_forward_train(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                    int64_t spatial, const float *scales, const float *biases, float *mean,
                                    float *variance, float *rolling_mean, float *rolling_variance, int act,
                                    dnb_stream stream);
/* Inference forward: batchnorm.forwardGpu else-branch (batchnorm.zig:147-152) + activate:
 * y = act(((x - rolling_mean) * (1/(sqrt(rolling_variance)+1e-6))) * scale + bias). */
dnb_status dnb_bn_act_forward_infer(const float *x, float *y, int64_t batch, int64_t filters, int64_t spatial,
                                    const float *scales, const float *biases, const float *rolling_mean,
                                    const float *rolling_variance, int act, dnb_stream stream);
/* Training forward from statistics that the producer of x computed (a convolution's GEMM
 * epilogue per output tile, say: convolutional.zig:239-270 runs the convolution and then
 * batchnorm.zig:129-153 reads its output twice, once for the statistics): pieces holds
 * npieces blocks laid out [piece][filters][3] = (count, mean, M2) of disjoint pieces of each
 * channel, fp64, with each channel's counts adding up to batch*spatial (pieces with count 0
 * are skipped). The pieces are merged in piece order (Chan's parallel variance), mean,
 * variance and the rolling statistics are written as by dnb_bn_act_forward_train, and
 * BN + activation are applied to x: one pass over x (8 bytes per element), no statistics
 * pass. No reference counterpart. */
dnb_status dnb_bn_act_forward_from_stats(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                         int64_t spatial, const double *pieces, int64_t npieces,
                                         const float *scales, const float *biases, float *mean, float *variance,
                                         float *rolling_mean, float *rolling_variance, int act,
                                         dnb_stream stream);
/* Backward through activation and batchnorm in one HBM pass: replaces gpu.gradientArray
 * (convolutional.zig:280) + batchnorm.backwardGpu (batchnorm.zig:155-169).
 *   x      the forward's input (l.x); delta = dL/dy (l.delta) on entry.
 *   y      optional forward output used for the activation gradient; NULL = recompute it
 *          from x, mean, variance, scales and biases with the forward's exact arithmetic.
 *   dx     out: dL/dx (the reference overwrites l.delta; dx may alias delta).
 *   bias_updates, scale_updates  in/out: += sum(g), += sum(g * x_norm), g = delta*act'(y).
 *   mean_delta, variance_delta   out (blas.zig:148-178 on delta*scales).
 * mean/variance are the statistics the forward normalised with (batch stats when
 * training, rolling ones at inference: batchnorm.zig:159-160). */
dnb_status dnb_bn_act_backward(const float *x, const float *y, const float *delta, float *dx, int64_t batch,
                               int64_t filters, int64_t spatial, const float *scales, const float *biases,
                               const float *mean, const float *variance, float *bias_updates, float *scale_updates,
                               float *mean_delta, float *variance_delta, int act, dnb_stream stream);
/* SGD with momentum and decay in one pass: replaces the weight part of
 * convolutional.updateGpu (convolutional.zig:332-334):
 *   wu += (-decay*batch) * w;  w += (learning_rate/batch) * wu;  wu *= momentum
 * with the two axpys each a single fused rounding, as blas.axpy. learning_rate already
 * includes the layer's learning_rate_scale. */
dnb_status dnb_sgd_momentum(int64_t n, float *weights, float *weight_updates, float learning_rate, float momentum,
                            float decay, int64_t batch, dnb_stream stream);
/* softmax + cross entropy + loss sum in one kernel: replaces misc.forwardSoftmaxGpu
 * (misc.zig:59-72) for groups = 1, stride = 1: output = softmax(input / temp) per row of n;
 * err = truth != 0 ? -log(output) : 0; delta = truth - output; *cost = sum(err) (the
 * reference pulls err to the host and sums it, misc.zig:66-70). cost is a device pointer
 * to one float; it may be NULL. */
dnb_status dnb_softmax_xent(const float *input, const float *truth, int64_t n, int64_t batch, float temp,
                            float *output, float *delta, float *err, float *cost, dnb_stream stream);

/* dnb_mean without any device allocation. No counterpart in the reference: it exists for
 * callers that may not call cudaMalloc on this path (a pre-budgeted memory pool or arena,
 * a fixed memory plan between its creation and its replay, a runtime that owns the
 * allocator). Same result as dnb_mean; its partial sums live in a fixed 1 MiB array inside
 * the library, held by every GPU that loads it. Limit: filters * ceil(batch*spatial/32768)
 * <= 262144, else DNB_ERR_UNSUPPORTED. The first call on a device looks up that array's
 * address; make it before any stream capture. Calls share the array: calls that overlap on
 * the GPU race, so serialise them. */
dnb_status dnb_mean_noalloc(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out,
                            dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* fused sync-BN across GPUs: no counterpart in the reference (it trains on one GPU); the  */
/* data-parallel form of the fused batchnorm entries, the statistics exchanged inside the  */
/* kernel over NVLink peer memory                                                          */
/* ------------------------------------------------------------------------------------ */

/* One process (or thread) per GPU, `world` ranks (<= 8). On the rank's device: allocates this
 * rank's exchange buffer for up to `max_channels` channels and writes its CUDA IPC handle
 * (64 bytes) to handle_out. The caller passes every rank's handle, in rank order, to
 * dnb_comm_connect on every rank (any host transport). */
dnb_status dnb_comm_init(int rank, int world, int64_t max_channels, void *handle_out, dnb_comm *comm);
/* Opens the peers' buffers (handles: world x 64 bytes, rank order). */
dnb_status dnb_comm_connect(dnb_comm comm, const void *handles);
dnb_status dnb_comm_destroy(dnb_comm comm);
/* dnb_bn_act_forward_train with the statistics of the whole data-parallel batch: every rank
 * passes its shard (the same batch, filters and spatial on every rank) and gets identical
 * mean, variance and rolling statistics. Every rank must make the same sequence of fused
 * sync-BN calls on a communicator, from one host thread per rank. Needs 16-byte aligned
 * tensors and filters <= max_channels, and spatial % 4 == 0 or an element count that is a
 * multiple of 4; DNB_ERR_UNSUPPORTED otherwise (the split entries below then apply). A rank that never makes its call leaves the others'
 * kernels waiting until the wait limit; they return DNB_ERR_TIMEOUT. The records a call
 * exchanges are tagged with its call number, which repeats after 2^32 - 1 fused calls on one
 * communicator: recreate the communicator before then. */
dnb_status dnb_syncbn_act_forward_train(dnb_comm comm, const float *x, float *y, float *x_norm, int64_t batch,
                                        int64_t filters, int64_t spatial, const float *scales, const float *biases,
                                        float *mean, float *variance, float *rolling_mean,
                                        float *rolling_variance, int act, dnb_stream stream);
/* dnb_bn_act_backward with sums over the whole data-parallel batch (normalize_delta divides
 * by batch*spatial*world). Same rules as dnb_syncbn_act_forward_train. */
dnb_status dnb_syncbn_act_backward(dnb_comm comm, const float *x, const float *y, const float *delta, float *dx,
                                   int64_t batch, int64_t filters, int64_t spatial, const float *scales,
                                   const float *biases, const float *mean, const float *variance,
                                   float *bias_updates, float *scale_updates, float *mean_delta,
                                   float *variance_delta, int act, dnb_stream stream);

/* ------------------------------------------------------------------------------------ */
/* data-parallel weight update: no counterpart in the reference (it trains on one GPU);    */
/* convolutional.zig:330-334's update with every rank's gradients summed, in one kernel    */
/* per rank over NVLink peer memory (reduce-scatter, fused SGD on the rank's shard and     */
/* all-gather, element by element)                                                         */
/* ------------------------------------------------------------------------------------ */

/* One process (or thread) per GPU, `world` ranks (<= 8), every rank the same n. Allocates this
 * rank's weight vector and gradient buffer (n floats each, padded; zero-filled) in one buffer
 * shared with the other ranks, writes its CUDA IPC handle (64 bytes) to handle_out, and returns
 * the two vectors and this rank's shard [*shard_lo, *shard_lo + *shard_n) of the weights. The
 * caller keeps its layer's weights and accumulates its gradients in them, and passes every
 * rank's handle, in rank order, to dnb_dpsgd_connect on every rank (any host transport). */
dnb_status dnb_dpsgd_init(int rank, int world, int64_t n, void *handle_out, float **weights, float **grads,
                          int64_t *shard_lo, int64_t *shard_n, dnb_dpsgd *group);
/* Opens the peers' buffers (handles: world x 64 bytes, rank order). */
dnb_status dnb_dpsgd_connect(dnb_dpsgd group, const void *handles);
/* One update on every rank: for this rank's shard, gradient = sum over ranks (rank order) of
 * their gradient vectors, momentum += gradient, then convolutional.zig:330-334 with batch the
 * global batch, and the new weights stored into every rank's weight vector. `momentum` is this
 * rank's shard of weight_updates (*shard_n floats, 16-byte aligned, zero before the first
 * step). Every rank must make the same calls; on return of the stream work every rank holds
 * identical weights, and the gradient vectors may be overwritten. A rank that never calls
 * leaves the others waiting until the wait limit (DNB_ERR_TIMEOUT from
 * dnb_check_device_error); recreate the group on every rank then. */
dnb_status dnb_dpsgd_step(dnb_dpsgd group, float *momentum, float learning_rate, float momentum_coef, float decay,
                          int64_t batch, dnb_stream stream);
dnb_status dnb_dpsgd_destroy(dnb_dpsgd group);

/* ------------------------------------------------------------------------------------ */
/* sync-BN across GPUs (the reference has no multi-GPU support, README.md:313-317).        */
/* Split form for a caller that owns the collective (e.g. NCCL): each rank computes its    */
/* per-channel partials, the caller combines them across ranks, then each rank applies.    */
/* ------------------------------------------------------------------------------------ */

/* Forward statistics of this rank's shard: partials[2*c] = mean_c and partials[2*c+1] =
 * M2_c (sum of squared deviations from mean_c) over batch*spatial elements, fp64. */
dnb_status dnb_syncbn_forward_partials(const float *x, int64_t batch, int64_t filters, int64_t spatial,
                                       double *partials, dnb_stream stream);
/* Combines `ranks` blocks of forward partials laid out [rank][filters][2] (as gathered by
 * an all-gather; every rank holds batch_per_rank*spatial elements per channel), writes
 * mean/variance/rolling stats exactly as dnb_bn_act_forward_train, and applies BN +
 * activation to this rank's x. */
dnb_status dnb_syncbn_forward_apply(const float *x, float *y, float *x_norm, int64_t batch, int64_t filters,
                                    int64_t spatial, const double *gathered, int ranks, const float *scales,
                                    const float *biases, float *mean, float *variance, float *rolling_mean,
                                    float *rolling_variance, int act, dnb_stream stream);
/* Backward sums of this rank's shard: partials[2*c] = sum(g), partials[2*c+1] =
 * sum(g*(x-mean)), g = delta*act'(y), fp64. Combine across ranks with a SUM all-reduce. */
dnb_status dnb_syncbn_backward_partials(const float *x, const float *y, const float *delta, int64_t batch,
                                        int64_t filters, int64_t spatial, const float *scales, const float *biases,
                                        const float *mean, const float *variance, int act, double *partials,
                                        dnb_stream stream);
/* Applies the backward with the all-reduced sums; total_count = global batch*spatial. */
dnb_status dnb_syncbn_backward_apply(const float *x, const float *y, const float *delta, float *dx, int64_t batch,
                                     int64_t filters, int64_t spatial, int64_t total_count, const double *reduced,
                                     const float *scales, const float *biases, const float *mean,
                                     const float *variance, float *bias_updates, float *scale_updates,
                                     float *mean_delta, float *variance_delta, int act, dnb_stream stream);

#ifdef __cplusplus
}
#endif
#endif /* DNB200_H */
