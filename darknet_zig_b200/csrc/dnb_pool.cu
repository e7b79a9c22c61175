// Pooling: maxpool with argmax indices forward and backward (pooling.zig:59-103,
// darknet_kernels.hip:472-539) and global average pooling forward
// (pooling.zig:146-158, darknet_kernels.hip:541-549).
#include <float.h>

#include <atomic>

#include "dnb_common.cuh"

namespace dnb {
namespace {

constexpr int kThreads = 256;

// pooling.zig:59-93: offset -pad/2, taps outside the image are skipped, strict '>' so the
// first maximum in (row, col) tap order wins; the index is the flat input index or -1.
// One thread per output; a warp's 32 outputs read contiguous 2*32-float runs of each
// input row, so the loads coalesce. SIZE > 0 fixes the window size at compile time.
template <int SIZE>
__global__ void __launch_bounds__(kThreads) k_maxpool_fwd(int64_t out_n, int in_h, int in_w, int out_h, int out_w,
                                                          int stride, int size_rt, int off, FastDiv fw, FastDiv fh,
                                                          bool fast, const float *__restrict__ in,
                                                          float *__restrict__ out, int32_t *__restrict__ idx) {
    const int size = SIZE > 0 ? SIZE : size_rt;
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x; id < out_n; id += step) {
        int64_t q;
        int i, j;
        if (fast) {
            uint32_t t, jj, ii;
            fw.divmod((uint32_t)id, t, jj);
            uint32_t qq;
            fh.divmod(t, qq, ii);
            q = qq;
            i = (int)ii;
            j = (int)jj;
        } else {
            j = (int)(id % out_w);
            const int64_t t = id / out_w;
            i = (int)(t % out_h);
            q = t / out_h;
        }
        const int64_t plane = q * (int64_t)in_h * in_w;
        float best = -FLT_MAX;
        int32_t best_i = -1;
        for (int n = 0; n < size; ++n) {
            const int ch = off + i * stride + n;
            if (ch < 0 || ch >= in_h) continue;
            for (int m = 0; m < size; ++m) {
                const int cw = off + j * stride + m;
                if (cw < 0 || cw >= in_w) continue;
                const int64_t index = plane + (int64_t)ch * in_w + cw;
                const float v = in[index];
                if (v > best) {
                    best = v;
                    best_i = (int32_t)index;
                }
            }
        }
        out[id] = best;
        idx[id] = best_i;
    }
}

// The darknet default 2x2 / stride 2 window (pad 1, so offset 0) on even images: every tap
// is inside the image, and two adjacent outputs read one 16-byte run of each of their two
// input rows. One thread per output pair; the taps are compared in the generic kernel's
// (row, col) order with the same strict '>', so values and indices are identical to it.
__global__ void __launch_bounds__(kThreads) k_maxpool_2x2(int64_t pairs, int in_w, int out_w, FastDiv fpw,
                                                          FastDiv foh, const float *__restrict__ in,
                                                          float *__restrict__ out, int32_t *__restrict__ idx) {
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x; id < pairs; id += step) {
        uint32_t t, jp, q, i;
        fpw.divmod((uint32_t)id, t, jp);
        foh.divmod(t, q, i);
        const int64_t row0 = ((int64_t)q * (2 * foh.d) + 2 * i) * in_w + 4 * (int64_t)jp;
        const int64_t row1 = row0 + in_w;
        const float4 a = ld4(in + row0), b = ld4(in + row1);
        float2 best;
        int2 bi;
        {  // output 2 jp: taps (row0, 0), (row0, 1), (row1, 0), (row1, 1)
            float v = -FLT_MAX;
            int k = -1;
            if (a.x > v) { v = a.x; k = (int)row0; }
            if (a.y > v) { v = a.y; k = (int)row0 + 1; }
            if (b.x > v) { v = b.x; k = (int)row1; }
            if (b.y > v) { v = b.y; k = (int)row1 + 1; }
            best.x = v;
            bi.x = k;
        }
        {  // output 2 jp + 1
            float v = -FLT_MAX;
            int k = -1;
            if (a.z > v) { v = a.z; k = (int)row0 + 2; }
            if (a.w > v) { v = a.w; k = (int)row0 + 3; }
            if (b.z > v) { v = b.z; k = (int)row1 + 2; }
            if (b.w > v) { v = b.w; k = (int)row1 + 3; }
            best.y = v;
            bi.y = k;
        }
        const int64_t o = (int64_t)t * out_w + 2 * (int64_t)jp;
        *reinterpret_cast<float2 *>(out + o) = best;
        *reinterpret_cast<int2 *>(idx + o) = bi;
    }
}

// The same 2x2 / stride-2 window on images whose width is even but not a multiple of 4
// (14 x 14 at BASELINE config 2): one thread per output reads one 8-byte pair of each of
// its two input rows; the comparisons and their order are k_maxpool_2x2's.
__global__ void __launch_bounds__(kThreads) k_maxpool_2x2_pair(int64_t out_n, int in_w, FastDiv fow, FastDiv foh,
                                                               const float *__restrict__ in, float *__restrict__ out,
                                                               int32_t *__restrict__ idx) {
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x; id < out_n; id += step) {
        uint32_t t, j, q, i;
        fow.divmod((uint32_t)id, t, j);
        foh.divmod(t, q, i);
        const int64_t row0 = ((int64_t)q * (2 * foh.d) + 2 * i) * in_w + 2 * (int64_t)j;
        const int64_t row1 = row0 + in_w;
        const float2 a = *reinterpret_cast<const float2 *>(in + row0);
        const float2 b = *reinterpret_cast<const float2 *>(in + row1);
        float v = -FLT_MAX;
        int k = -1;
        if (a.x > v) { v = a.x; k = (int)row0; }
        if (a.y > v) { v = a.y; k = (int)row0 + 1; }
        if (b.x > v) { v = b.x; k = (int)row1; }
        if (b.y > v) { v = b.y; k = (int)row1 + 1; }
        out[id] = v;
        idx[id] = k;
    }
}

__device__ __forceinline__ int ceil_div_pos(int a, int b) { return a >= 0 ? (a + b - 1) / b : a / b; }

// pooling.zig:95-103 as a gather: input element `in` receives, in increasing output index,
// the deltas of every output whose index points at it -- the order the CPU scatter adds
// them in, so the result is bit-identical even with overlapping windows.
__global__ void __launch_bounds__(kThreads) k_maxpool_bwd(int64_t in_n, int in_h, int in_w, int out_h, int out_w,
                                                          int stride, int size, int off, const float *__restrict__ delta,
                                                          float *__restrict__ prev, const int32_t *__restrict__ idx) {
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t id = (int64_t)blockIdx.x * kThreads + threadIdx.x; id < in_n; id += step) {
        const int x = (int)(id % in_w);
        const int64_t t = id / in_w;
        const int y = (int)(t % in_h);
        const int64_t q = t / in_h;
        // outputs (i, j) whose window covers (y, x): off + i*stride <= y < off + i*stride + size
        int i0 = ceil_div_pos(y - off - size + 1, stride), i1 = (y - off) / stride;
        int j0 = ceil_div_pos(x - off - size + 1, stride), j1 = (x - off) / stride;
        if (i0 < 0) i0 = 0;
        if (j0 < 0) j0 = 0;
        if (i1 > out_h - 1) i1 = out_h - 1;
        if (j1 > out_w - 1) j1 = out_w - 1;
        float v = prev[id];
        for (int i = i0; i <= i1; ++i) {
            for (int j = j0; j <= j1; ++j) {
                const int64_t o = (q * out_h + i) * out_w + j;
                if ((int64_t)idx[o] == id) v = v + delta[o];
            }
        }
        prev[id] = v;
    }
}

// pooling.zig:146-158. A block of kAvgThreads threads stages PB consecutive planes (PB*S
// floats, contiguous) in shared memory with coalesced 128-bit loads; thread t then sums
// plane t in order, exactly as the CPU loop does, so the output is bit-identical. The planes
// are read once. Small blocks with small tiles let an SM keep many tiles in flight.
constexpr int kAvgThreads = 64;
__global__ void __launch_bounds__(kAvgThreads) k_avgpool_fwd(int64_t planes, int S, int PB, bool vec,
                                                          const float *__restrict__ in, float *__restrict__ out) {
    extern __shared__ __align__(16) float tile[];
    const float denom = (float)S;
    for (int64_t q0 = (int64_t)blockIdx.x * PB; q0 < planes; q0 += (int64_t)gridDim.x * PB) {
        const int np = (int)(planes - q0 < PB ? planes - q0 : PB);
        const int64_t base = q0 * S;
        const int nf = np * S;
        __syncthreads();
        if (vec) {
            const int nf4 = nf >> 2;
            const float4 *src = reinterpret_cast<const float4 *>(in + base);
            for (int k = threadIdx.x; k < nf4; k += kAvgThreads) reinterpret_cast<float4 *>(tile)[k] = __ldcs(src + k);
            for (int k = (nf4 << 2) + threadIdx.x; k < nf; k += kAvgThreads) tile[k] = in[base + k];
        } else {
            for (int k = threadIdx.x; k < nf; k += kAvgThreads) tile[k] = in[base + k];
        }
        __syncthreads();
        for (int t = threadIdx.x; t < np; t += kAvgThreads) {
            const float *row = tile + (int64_t)t * S;
            float sum = 0.0f;
            for (int s = 0; s < S; ++s) sum += row[s];
            out[q0 + t] = sum / denom;
        }
    }
}

// Large planes: one warp per plane, shuffle tree (not the CPU's summation order).
__global__ void k_avgpool_fwd_warp(int64_t planes, int64_t S, const float *__restrict__ in, float *__restrict__ out) {
    const int lane = threadIdx.x & 31;
    const int64_t wpb = blockDim.x >> 5;
    for (int64_t q = (int64_t)blockIdx.x * wpb + (threadIdx.x >> 5); q < planes; q += (int64_t)gridDim.x * wpb) {
        float sum = 0.0f;
        for (int64_t s = lane; s < S; s += 32) sum += in[q * S + s];
        sum = warp_sum(sum);
        if (lane == 0) out[q] = sum / (float)S;
    }
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_forward_maxpool(int64_t out_n, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride, int64_t size,
                               int64_t pad, const float *input, float *output, int32_t *indexes, dnb_stream stream) {
    if (out_n < 0 || in_h <= 0 || in_w <= 0 || in_c <= 0 || stride <= 0 || size <= 0 || pad < 0)
        return fail(DNB_ERR_INVALID, "forward_maxpool: bad shape");
    if (in_h > INT32_MAX / 2 || in_w > INT32_MAX / 2) return fail(DNB_ERR_UNSUPPORTED, "forward_maxpool: too large");
    const int64_t out_h = (in_h + pad - size) / stride + 1, out_w = (in_w + pad - size) / stride + 1;  // pooling.zig:33
    if (out_h <= 0 || out_w <= 0) return fail(DNB_ERR_INVALID, "forward_maxpool: window larger than the image");
    if (out_n % (out_h * out_w) != 0) return fail(DNB_ERR_INVALID, "forward_maxpool: out_n is not batch*c*out_h*out_w");
    if (out_n == 0) return DNB_OK;
    if (!input || !output || !indexes) return fail(DNB_ERR_INVALID, "forward_maxpool: null pointer");
    if ((out_n / (out_h * out_w)) * in_h * in_w > (int64_t)INT32_MAX)
        return fail(DNB_ERR_UNSUPPORTED, "forward_maxpool: int32 indexes cannot address the input");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    const bool fast = out_n < (1ll << 32);
    const FastDiv fw((uint32_t)out_w), fh((uint32_t)out_h);
    const int off = -(int)(pad / 2);
    const unsigned grid = grid_for(out_n, kThreads, ds);
    if (size == 2 && stride == 2 && off == 0 && in_h == 2 * out_h && in_w == 2 * out_w && in_w % 4 == 0 && fast &&
        aligned16(input) && (reinterpret_cast<uintptr_t>(output) & 7u) == 0 &&
        (reinterpret_cast<uintptr_t>(indexes) & 7u) == 0) {
        const int64_t pairs = out_n / 2;
        k_maxpool_2x2<<<grid_for(pairs, kThreads, ds), kThreads, 0, s>>>(
            pairs, (int)in_w, (int)out_w, FastDiv((uint32_t)(out_w / 2)), FastDiv((uint32_t)out_h), input, output,
            indexes);
    } else if (size == 2 && stride == 2 && off == 0 && in_h == 2 * out_h && in_w == 2 * out_w && fast &&
               (reinterpret_cast<uintptr_t>(input) & 7u) == 0) {
        k_maxpool_2x2_pair<<<grid, kThreads, 0, s>>>(out_n, (int)in_w, FastDiv((uint32_t)out_w),
                                                     FastDiv((uint32_t)out_h), input, output, indexes);
    } else if (size == 2)
        k_maxpool_fwd<2><<<grid, kThreads, 0, s>>>(out_n, (int)in_h, (int)in_w, (int)out_h, (int)out_w, (int)stride, 2,
                                                   off, fw, fh, fast, input, output, indexes);
    else if (size == 3)
        k_maxpool_fwd<3><<<grid, kThreads, 0, s>>>(out_n, (int)in_h, (int)in_w, (int)out_h, (int)out_w, (int)stride, 3,
                                                   off, fw, fh, fast, input, output, indexes);
    else
        k_maxpool_fwd<0><<<grid, kThreads, 0, s>>>(out_n, (int)in_h, (int)in_w, (int)out_h, (int)out_w, (int)stride,
                                                   (int)size, off, fw, fh, fast, input, output, indexes);
    return after_launch(s, "forward_maxpool");
}

dnb_status dnb_backward_maxpool(int64_t in_n, int64_t in_h, int64_t in_w, int64_t in_c, int64_t stride, int64_t size,
                                int64_t pad, const float *delta, float *prev_delta, const int32_t *indexes,
                                dnb_stream stream) {
    if (in_n < 0 || in_h <= 0 || in_w <= 0 || in_c <= 0 || stride <= 0 || size <= 0 || pad < 0)
        return fail(DNB_ERR_INVALID, "backward_maxpool: bad shape");
    const int64_t out_h = (in_h + pad - size) / stride + 1, out_w = (in_w + pad - size) / stride + 1;
    if (out_h <= 0 || out_w <= 0) return fail(DNB_ERR_INVALID, "backward_maxpool: window larger than the image");
    if (in_n % (in_h * in_w) != 0) return fail(DNB_ERR_INVALID, "backward_maxpool: in_n is not batch*c*h*w");
    if (in_n == 0) return DNB_OK;
    if (!delta || !prev_delta || !indexes) return fail(DNB_ERR_INVALID, "backward_maxpool: null pointer");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    k_maxpool_bwd<<<grid_for(in_n, kThreads, ds), kThreads, 0, s>>>(in_n, (int)in_h, (int)in_w, (int)out_h,
                                                                    (int)out_w, (int)stride, (int)size,
                                                                    -(int)(pad / 2), delta, prev_delta, indexes);
    return after_launch(s, "backward_maxpool");
}

dnb_status dnb_forward_avgpool(int64_t n, int64_t w, int64_t h, int64_t c, const float *input, float *output,
                               dnb_stream stream) {
    if (n < 0 || w <= 0 || h <= 0 || c <= 0) return fail(DNB_ERR_INVALID, "forward_avgpool: bad shape");
    if (n == 0) return DNB_OK;
    if (!input || !output) return fail(DNB_ERR_INVALID, "forward_avgpool: null pointer");
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const cudaStream_t s = as_stream(stream);
    const int64_t S = w * h;
    // planes per block: a multiple of 4 (so a tile starts 16-byte aligned), at most one per
    // thread, with the tile within 16 KB of shared memory (96 KB for planes of more than 256
    // floats, so that a block still sums at least 4 planes in the CPU's order)
    const int64_t budget = S <= 256 ? 16 * 1024 : 96 * 1024;
    int64_t pb = budget / (S * 4);
    if (pb > kAvgThreads) pb = kAvgThreads;
    pb &= ~(int64_t)3;
    if (pb >= 4) {
        const size_t smem = (size_t)pb * S * sizeof(float);
        if (smem > 48 * 1024) {
            static std::atomic<int> big[kMaxDevices];
            if (!big[ds->device].load(std::memory_order_relaxed)) {
                DNB_CUDA(cudaFuncSetAttribute(k_avgpool_fwd, cudaFuncAttributeMaxDynamicSharedMemorySize, 96 * 1024));
                big[ds->device].store(1, std::memory_order_relaxed);
            }
        }
        const int64_t blocks = (n + pb - 1) / pb;
        const int64_t cap = (int64_t)ds->sm_count * 32;
        const unsigned grid = (unsigned)(blocks < cap ? blocks : cap);
        k_avgpool_fwd<<<grid, kAvgThreads, smem, s>>>(n, (int)S, (int)pb, aligned16(input), input, output);
    } else {
        k_avgpool_fwd_warp<<<grid_for(n * 32, kThreads, ds), kThreads, 0, s>>>(n, S, input, output);
    }
    return after_launch(s, "forward_avgpool");
}

}  // extern "C"
