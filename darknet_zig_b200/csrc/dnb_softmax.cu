// Softmax and cross entropy: blas.zig:213-252 (softmax_kernel / softmax_x_ent_kernel,
// darknet_kernels.hip:350-379) and the softmax layer's forward (misc.zig:41-72).
//
// The reference's softmax kernel gives each row to ONE thread, which walks the row three
// times serially (darknet_kernels.hip:350-360): 256 threads for the whole classifier head.
// Here a warp owns a row: shuffle max, exp + shuffle sum, divide. The per-element
// arithmetic is the CPU's (exp(x/temp - largest/temp), then e/sum); the sum is a tree.
#include <float.h>

#include <atomic>

#include "dnb_common.cuh"

namespace dnb {
namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;

__device__ __forceinline__ float row_softmax(const float *in, float *out, int64_t n, int64_t stride, float temp,
                                             int lane) {
    float largest = -FLT_MAX;  // blas.zig:214
    for (int64_t i = lane; i < n; i += 32) {
        const float v = in[i * stride];
        largest = v > largest ? v : largest;
    }
    largest = warp_max(largest);
    float sum = 0.0f;
    for (int64_t i = lane; i < n; i += 32) {
        const float e = expf(in[i * stride] / temp - largest / temp);
        sum += e;
        out[i * stride] = e;
    }
    sum = warp_sum(sum);
    __syncwarp();
    for (int64_t i = lane; i < n; i += 32) out[i * stride] = out[i * stride] / sum;
    return sum;
}

// blas.zig:225-242: row q = (b, g) starts at b*batch_offset + g*group_offset
__global__ void __launch_bounds__(kThreads) k_softmax(const float *in, int64_t n, int64_t batch, int64_t batch_offset,
                                                      int64_t groups, int64_t group_offset, int64_t stride,
                                                      float temp, float *out) {
    const int lane = threadIdx.x & 31;
    const int64_t rows = batch * groups;
    for (int64_t q = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); q < rows; q += (int64_t)gridDim.x * kWarps) {
        const int64_t b = q / groups, g = q % groups;
        const int64_t off = b * batch_offset + g * group_offset;
        row_softmax(in + off, out + off, n, stride, temp, lane);
    }
}

// blas.zig:247-252 (no clamp of p: the CPU path takes -log(p) as is)
__global__ void __launch_bounds__(kThreads) k_xent(int64_t n, const float *pred, const float *truth, float *delta,
                                                   float *err) {
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t i = (int64_t)blockIdx.x * kThreads + threadIdx.x; i < n; i += step) {
        const float t = truth[i], p = pred[i];
        err[i] = t != 0.0f ? -logf(p) : 0.0f;
        delta[i] = t - p;
    }
}

// misc.zig:41-50 fused: softmax, cross entropy and the row's loss in one pass over the row.
__global__ void __launch_bounds__(kThreads) k_softmax_xent(const float *in, const float *truth, int64_t n,
                                                           int64_t batch, float temp, float *out, float *delta,
                                                           float *err, float *row_loss) {
    const int lane = threadIdx.x & 31;
    for (int64_t q = (int64_t)blockIdx.x * kWarps + (threadIdx.x >> 5); q < batch; q += (int64_t)gridDim.x * kWarps) {
        const int64_t off = q * n;
        row_softmax(in + off, out + off, n, 1, temp, lane);
        __syncwarp();
        float loss = 0.0f;
        for (int64_t i = lane; i < n; i += 32) {
            const float p = out[off + i], t = truth[off + i];
            const float e = t != 0.0f ? -logf(p) : 0.0f;
            err[off + i] = e;
            delta[off + i] = t - p;
            loss += e;
        }
        loss = warp_sum(loss);
        if (lane == 0 && row_loss) row_loss[q] = loss;
    }
}

// misc.zig:41-50 fused, one block per row with the row staged in shared memory (rows of up
// to kRowSmem floats): the row is read from HBM once, the max and the sum are block trees,
// and output, err and delta are written in one pass. A classifier head has few rows (256 at
// BASELINE config 3), so a warp per row leaves most of the GPU idle and walks each row
// three times through global memory; a block per row reads 1000 classes in 4 loads a thread.
constexpr int kRowSmem = 12288;  // floats of one staged row (48 KB)

__device__ __forceinline__ float block_max(float v, float *red) {
    v = warp_max(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = threadIdx.x < kWarps ? red[threadIdx.x] : -FLT_MAX;
    if (threadIdx.x < 32) t = warp_max(t);
    if (threadIdx.x == 0) red[kWarps] = t;
    __syncthreads();
    t = red[kWarps];
    __syncthreads();
    return t;
}
__device__ __forceinline__ float block_sum_f(float v, float *red) {
    v = warp_sum(v);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    float t = threadIdx.x < kWarps ? red[threadIdx.x] : 0.0f;
    if (threadIdx.x < 32) t = warp_sum(t);
    if (threadIdx.x == 0) red[kWarps] = t;
    __syncthreads();
    t = red[kWarps];
    __syncthreads();
    return t;
}

// With `cost`, the last block to finish (a counter in the stream's workspace, reset by that
// block) adds the row losses in fp64 in row order -- the same sum k_cost forms -- so the
// loss needs no second launch.
__device__ __forceinline__ void cost_sum(const float *row_loss, int64_t batch, float *cost) {
    __shared__ double part[32];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < batch; i += blockDim.x) s += (double)row_loss[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
        t = warp_sum(t);
        if (threadIdx.x == 0) *cost = (float)t;
    }
}

__global__ void __launch_bounds__(kThreads) k_softmax_xent_rows(const float *in, const float *truth, int64_t n,
                                                                int64_t batch, float temp, float *out, float *delta,
                                                                float *err, float *row_loss, float *cost,
                                                                unsigned *done) {
    extern __shared__ float row[];
    __shared__ float red[kWarps + 1];
    __shared__ int s_last;
    for (int64_t q = blockIdx.x; q < batch; q += gridDim.x) {
        const int64_t off = q * n;
        float largest = -FLT_MAX;  // blas.zig:214
        for (int64_t i = threadIdx.x; i < n; i += kThreads) {
            const float v = in[off + i];
            row[i] = v;
            largest = v > largest ? v : largest;
        }
        largest = block_max(largest, red);
        float sum = 0.0f;
        for (int64_t i = threadIdx.x; i < n; i += kThreads) {
            const float e = expf(row[i] / temp - largest / temp);  // blas.zig:218
            row[i] = e;
            sum += e;
        }
        sum = block_sum_f(sum, red);
        float loss = 0.0f;
        for (int64_t i = threadIdx.x; i < n; i += kThreads) {
            const float p = row[i] / sum;  // blas.zig:221
            const float t = truth[off + i];
            const float e = t != 0.0f ? -logf(p) : 0.0f;  // blas.zig:250
            out[off + i] = p;
            err[off + i] = e;
            delta[off + i] = t - p;  // blas.zig:251
            loss += e;
        }
        loss = block_sum_f(loss, red);
        if (threadIdx.x == 0 && row_loss) row_loss[q] = loss;
    }
    if (!cost) return;
    // this block's row losses, visible before it counts itself; the last block sums them all
    __threadfence();
    if (threadIdx.x == 0) s_last = atomicAdd(done, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    cost_sum(row_loss, batch, cost);
    if (threadIdx.x == 0) *done = 0u;  // for the next launch on this stream
}

// The cost: rows added in fp64 in row order by one block (deterministic).
__global__ void k_cost(const float *row_loss, int64_t batch, float *cost) {
    __shared__ double part[32];
    double s = 0.0;
    for (int64_t i = threadIdx.x; i < batch; i += blockDim.x) s += (double)row_loss[i];
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = s;
    __syncthreads();
    if (threadIdx.x < 32) {
        double t = threadIdx.x < (blockDim.x >> 5) ? part[threadIdx.x] : 0.0;
        t = warp_sum(t);
        if (threadIdx.x == 0) *cost = (float)t;
    }
}

unsigned rows_grid(int64_t rows, const DeviceState *ds) {
    int64_t blocks = (rows + kWarps - 1) / kWarps;
    const int64_t cap = (int64_t)ds->sm_count * 8;
    if (blocks > cap) blocks = cap;
    return (unsigned)(blocks < 1 ? 1 : blocks);
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_softmax(const float *input, int64_t n, int64_t batch, int64_t batch_offset, int64_t groups,
                       int64_t group_offset, int64_t stride, float temp, float *output, dnb_stream stream) {
    if (n < 0 || batch < 0 || groups < 0 || stride <= 0 || batch_offset < 0 || group_offset < 0)
        return fail(DNB_ERR_INVALID, "softmax: bad shape");
    if (n == 0 || batch == 0 || groups == 0) return DNB_OK;
    if (!input || !output) return fail(DNB_ERR_INVALID, "softmax: null pointer");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    k_softmax<<<rows_grid(batch * groups, ds), kThreads, 0, s>>>(input, n, batch, batch_offset, groups, group_offset,
                                                                 stride, temp, output);
    return after_launch(s, "softmax");
}

dnb_status dnb_softmax_cross_entropy(int64_t n, const float *pred, const float *truth, float *delta, float *err,
                                     dnb_stream stream) {
    if (n < 0) return fail(DNB_ERR_INVALID, "softmax_cross_entropy: negative size");
    if (n == 0) return DNB_OK;
    if (!pred || !truth || !delta || !err) return fail(DNB_ERR_INVALID, "softmax_cross_entropy: null pointer");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    k_xent<<<grid_for(n, kThreads, ds), kThreads, 0, s>>>(n, pred, truth, delta, err);
    return after_launch(s, "softmax_cross_entropy");
}

dnb_status dnb_softmax_xent(const float *input, const float *truth, int64_t n, int64_t batch, float temp,
                            float *output, float *delta, float *err, float *cost, dnb_stream stream) {
    if (n < 0 || batch < 0) return fail(DNB_ERR_INVALID, "softmax_xent: negative size");
    if (n == 0 || batch == 0) return DNB_OK;
    if (!input || !truth || !output || !delta || !err) return fail(DNB_ERR_INVALID, "softmax_xent: null pointer");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    float *row_loss = nullptr;
    if (cost) {
        Workspace *ws = nullptr;
        DNB_TRY(workspace(s, sizeof(float) * (size_t)batch, &ws));
        row_loss = static_cast<float *>(ws->scratch);
    }
    if (n <= kRowSmem) {
        // the per-device attribute for rows beyond the default 48 KB, set once to the most
        // a staged row takes
        const size_t smem = sizeof(float) * (size_t)n;
        if (smem > 48 * 1024) {
            static std::atomic<int> big[kMaxDevices];
            if (!big[ds->device].load(std::memory_order_relaxed)) {
                DNB_CUDA(cudaFuncSetAttribute(k_softmax_xent_rows, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                              (int)(sizeof(float) * kRowSmem)));
                big[ds->device].store(1, std::memory_order_relaxed);
            }
        }
        const int64_t cap = (int64_t)ds->sm_count * 8;
        const unsigned grid = (unsigned)(batch < cap ? batch : cap);
        Workspace *ws = nullptr;
        unsigned *done = nullptr;
        if (cost) {
            DNB_TRY(workspace(s, sizeof(float) * (size_t)batch, &ws));
            done = ws->sync + kSyncSoftmaxDone;
        }
        k_softmax_xent_rows<<<grid, kThreads, smem, s>>>(input, truth, n, batch, temp, output, delta, err, row_loss,
                                                         cost, done);
        return after_launch(s, "softmax_xent");
    }
    k_softmax_xent<<<rows_grid(batch, ds), kThreads, 0, s>>>(input, truth, n, batch, temp, output, delta, err,
                                                             row_loss);
    DNB_TRY(after_launch(s, "softmax_xent"));
    if (cost) {
        k_cost<<<1, 1024, 0, s>>>(row_loss, batch, cost);
        DNB_TRY(after_launch(s, "softmax_xent cost"));
    }
    return DNB_OK;
}

}  // extern "C"
