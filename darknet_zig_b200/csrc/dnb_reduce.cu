// Standalone per-channel reductions: blas.zig:73-100 (backward_bias, backward_scale) and
// blas.zig:106-178 (mean, variance, mean_delta, variance_delta), each the replacement of
// one reference kernel that ran a single 256-thread block per channel
// (darknet_kernels.hip:227-333, launched by gpu.zig:474-477).
//
// Two deterministic stages. Stage 1: a grid of (chunk, channel) blocks; each block sums
// its chunk of one channel's batch*spatial elements (128-bit loads when a plane is a
// multiple of 4 floats) into one fp32 partial. Stage 2: one warp per channel adds the
// chunk partials in fp64 in a fixed order and applies the op's closing formula. The
// result does not depend on scheduling, and the fp64 combine keeps the fp32 error to the
// per-block sums (well inside the 1e-5 relative bar at every BASELINE size).
#include "dnb_common.cuh"

namespace dnb {
namespace {

constexpr int kThreads = 256;
constexpr int64_t kChunkElems = 32768;  // elements one stage-1 block reduces

// Per-element terms. Each op reads one or two tensors at the same element offset.
struct TermSum {  // sum(a)
    __device__ float operator()(float a, float, float) const { return a; }
};
struct TermProd {  // sum(a*b)
    __device__ float operator()(float a, float b, float) const { return a * b; }
};
struct TermSqDev {  // sum((a-m)^2)
    __device__ float operator()(float a, float, float m) const {
        float d = a - m;
        return d * d;
    }
};
struct TermProdDev {  // sum(b*(a-m)) -- a = x, b = delta (blas.zig:174)
    __device__ float operator()(float a, float b, float m) const { return b * (a - m); }
};

struct Geometry {
    int64_t batch, filters, spatial;
    int64_t per_channel;  // batch*spatial
    int64_t chunk;        // elements per block (a multiple of 4 when vec)
    int chunks;
    bool vec;             // spatial % 4 == 0 and both tensors 16-byte aligned
    FastDiv fs4;          // divides a float4 index by spatial/4
    FastDiv fs;           // divides an element index by spatial
    bool fast;            // per-channel index space fits 32 bits
};

// Stage 1: block (chunk, c) -> partial[c * chunks + chunk].
template <class Term, bool TWO>
__global__ void __launch_bounds__(kThreads) k_chan_partial(Geometry g, const float *a, const float *b,
                                                         const float *mvec, float *partial) {
    __shared__ float red[32];
    const int64_t c = blockIdx.y;
    const int64_t k0 = (int64_t)blockIdx.x * g.chunk;
    int64_t k1 = k0 + g.chunk;
    if (k1 > g.per_channel) k1 = g.per_channel;
    const float m = mvec ? mvec[c] : 0.0f;
    const int64_t cs = g.filters * g.spatial;  // stride between planes of one channel
    const Term term;
    float acc = 0.0f;
    if (g.vec) {
        const int64_t s4 = g.spatial >> 2;
        for (int64_t k = (k0 >> 2) + threadIdx.x; k < (k1 >> 2); k += kThreads) {
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
            const int64_t off = n * cs + c * g.spatial + 4 * r;
            const float4 va = ld4(a + off);
            const float4 vb = TWO ? ld4(b + off) : va;
            acc += term(va.x, vb.x, m);
            acc += term(va.y, vb.y, m);
            acc += term(va.z, vb.z, m);
            acc += term(va.w, vb.w, m);
        }
    } else {
        for (int64_t k = k0 + threadIdx.x; k < k1; k += kThreads) {
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
            const int64_t off = n * cs + c * g.spatial + r;
            const float va = a[off];
            const float vb = TWO ? b[off] : va;
            acc += term(va, vb, m);
        }
    }
    const float total = block_sum<kThreads>(acc, red);
    if (threadIdx.x == 0) partial[c * g.chunks + blockIdx.x] = total;
}

enum class Close { AccumulateInto, Mean, Variance, MeanDelta, VarianceDelta };

// Stage 2: one warp per channel.
__global__ void k_chan_close(int64_t filters, int chunks, const float *partial, Close how, float scale,
                             const float *var, float *out) {
    const int64_t c = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (c >= filters) return;
    double s = 0.0;
    for (int i = lane; i < chunks; i += 32) s += (double)partial[c * chunks + i];
    s = warp_sum(s);
    if (lane != 0) return;
    const float sum = (float)s;
    switch (how) {
    case Close::AccumulateInto: out[c] += sum; break;                       // blas.zig:79,98
    case Close::Mean: out[c] = sum * scale; break;                          // blas.zig:114
    case Close::Variance: out[c] = sum * scale; break;                      // blas.zig:133
    case Close::MeanDelta: out[c] = sum * (-1.0f / sqrtf(var[c] + 0.00001f)); break;  // blas.zig:155
    case Close::VarianceDelta:                                               // blas.zig:176
        out[c] = sum * -0.5f * powf(var[c] + 0.00001f, -1.5f);
        break;
    }
}

template <class Term, bool TWO>
dnb_status chan_reduce(const float *a, const float *b, const float *mvec, int64_t batch, int64_t filters,
                       int64_t spatial, Close how, float scale, const float *var, float *out, cudaStream_t stream,
                       const char *what) {
    if (batch < 0 || filters < 0 || spatial < 0) return fail(DNB_ERR_INVALID, "%s: negative size", what);
    if (filters == 0) return DNB_OK;
    if (!out || (batch * spatial > 0 && (!a || (TWO && !b)))) return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    if (filters > 65535) return fail(DNB_ERR_UNSUPPORTED, "%s: more than 65535 channels", what);
    Geometry g;
    g.batch = batch;
    g.filters = filters;
    g.spatial = spatial;
    g.per_channel = batch * spatial;
    g.vec = spatial % 4 == 0 && aligned16(a) && (!TWO || aligned16(b));
    g.chunk = kChunkElems;
    int64_t chunks = (g.per_channel + g.chunk - 1) / g.chunk;
    if (chunks < 1) chunks = 1;
    g.chunks = (int)chunks;
    g.fast = g.per_channel < (1ll << 32);
    if (spatial > 0) {
        g.fs = FastDiv((uint32_t)(g.fast ? spatial : 1));
        g.fs4 = FastDiv((uint32_t)(g.fast && g.vec ? spatial / 4 : 1));
    }
    Workspace *ws = nullptr;
    DNB_TRY(workspace(stream, sizeof(float) * (size_t)(filters * chunks), &ws));
    float *partial = static_cast<float *>(ws->scratch);
    if (g.per_channel > 0) {
        k_chan_partial<Term, TWO><<<dim3((unsigned)chunks, (unsigned)filters), kThreads, 0, stream>>>(g, a, b, mvec,
                                                                                                     partial);
    } else {
        DNB_CUDA(cudaMemsetAsync(partial, 0, sizeof(float) * (size_t)(filters * chunks), stream));
    }
    DNB_TRY(after_launch(stream, what));
    const unsigned warps_per_block = 8;
    const unsigned blocks = (unsigned)((filters + warps_per_block - 1) / warps_per_block);
    k_chan_close<<<blocks, 32 * warps_per_block, 0, stream>>>(filters, g.chunks, partial, how, scale, var, out);
    return after_launch(stream, what);
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_backward_bias(float *bias_updates, const float *delta, int64_t batch, int64_t filters, int64_t spatial,
                             dnb_stream stream) {
    return chan_reduce<TermSum, false>(delta, nullptr, nullptr, batch, filters, spatial, Close::AccumulateInto, 1.0f,
                                       nullptr, bias_updates, as_stream(stream), "backward_bias");
}

dnb_status dnb_backward_scale(const float *x_norm, const float *delta, int64_t batch, int64_t filters,
                              int64_t spatial, float *scale_updates, dnb_stream stream) {
    return chan_reduce<TermProd, true>(x_norm, delta, nullptr, batch, filters, spatial, Close::AccumulateInto, 1.0f,
                                       nullptr, scale_updates, as_stream(stream), "backward_scale");
}

dnb_status dnb_mean(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out, dnb_stream stream) {
    const float scale = 1.0f / (float)(batch * spatial);  // blas.zig:107
    return chan_reduce<TermSum, false>(x, nullptr, nullptr, batch, filters, spatial, Close::Mean, scale, nullptr, out,
                                       as_stream(stream), "mean");
}

dnb_status dnb_variance(const float *x, const float *mean, int64_t batch, int64_t filters, int64_t spatial, float *out,
                        dnb_stream stream) {
    if (filters > 0 && !mean) return fail(DNB_ERR_INVALID, "variance: mean is null");
    const float scale = 1.0f / (float)(batch * spatial - 1);  // blas.zig:122
    return chan_reduce<TermSqDev, false>(x, nullptr, mean, batch, filters, spatial, Close::Variance, scale, nullptr,
                                         out, as_stream(stream), "variance");
}

dnb_status dnb_mean_delta(const float *delta, const float *variance, int64_t batch, int64_t filters, int64_t spatial,
                          float *out, dnb_stream stream) {
    if (filters > 0 && !variance) return fail(DNB_ERR_INVALID, "mean_delta: variance is null");
    return chan_reduce<TermSum, false>(delta, nullptr, nullptr, batch, filters, spatial, Close::MeanDelta, 1.0f,
                                       variance, out, as_stream(stream), "mean_delta");
}

dnb_status dnb_variance_delta(const float *x, const float *delta, const float *mean, const float *variance,
                              int64_t batch, int64_t filters, int64_t spatial, float *out, dnb_stream stream) {
    if (filters > 0 && (!mean || !variance)) return fail(DNB_ERR_INVALID, "variance_delta: null pointer");
    return chan_reduce<TermProdDev, true>(x, delta, mean, batch, filters, spatial, Close::VarianceDelta, 1.0f,
                                          variance, out, as_stream(stream), "variance_delta");
}

}  // extern "C"

#include <mutex>

// --------------------------------------------------------------------------------------
// dnb_mean_noalloc: dnb_mean for callers that must not allocate device memory.
//
// Some hosts cannot call cudaMalloc on the path that computes batch statistics: code that
// runs inside a pre-sized memory pool or arena (where every byte is budgeted up front),
// code between the creation and the replay of a fixed memory plan, or a foreign runtime
// that owns the device allocator. dnb_mean itself may grow the library's per-stream
// workspace on first use; this variant keeps its per-(channel, chunk) partial sums in a
// fixed array compiled into the library instead, and otherwise runs the same two kernels.
//
// The array is a file-scope __device__ object: every GPU that loads the library holds it
// (kNoAllocScratchFloats floats, 1 MiB) until the process exits. Host code may not pass
// the array's name to a kernel -- on the host that name is only a stand-in -- so the first
// call on each device looks the device address up with cudaGetSymbolAddress (that device
// current) and caches it; make that first call before any stream capture. Every call
// shares the array and it keeps the last call's partials, so calls that overlap on the GPU
// (two streams, or two host threads) race; serialise them. Requests needing more than
// kNoAllocScratchFloats partials (filters * ceil(batch*spatial / 32768)) are rejected.
// --------------------------------------------------------------------------------------

namespace dnb {
namespace {

constexpr int64_t kNoAllocScratchFloats = 1 << 18;
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats];

constexpr int kNoAllocMaxDevices = 64;
float *g_noalloc_ptr[kNoAllocMaxDevices] = {};
std::once_flag g_noalloc_once[kNoAllocMaxDevices];
cudaError_t g_noalloc_err[kNoAllocMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
dnb_status noalloc_scratch(float **out) {
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    if (device < 0 || device >= kNoAllocMaxDevices)
        return fail(DNB_ERR_UNSUPPORTED, "mean_noalloc: device %d beyond %d", device, kNoAllocMaxDevices);
    std::call_once(g_noalloc_once[device], [device] {
        void *p = nullptr;
        g_noalloc_err[device] = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (g_noalloc_err[device] == cudaSuccess) g_noalloc_ptr[device] = static_cast<float *>(p);
    });
    if (g_noalloc_err[device] != cudaSuccess)
        return cuda_fail(g_noalloc_err[device], "cudaGetSymbolAddress(g_noalloc_scratch)", __FILE__, __LINE__);
    *out = g_noalloc_ptr[device];
    return DNB_OK;
}

// after_launch without its device lookup: counts the launch, checks it, and under
// dnb_set_sync_after_launch(1) synchronises the stream and reports a fault here (the
// device-side wait word is not read: these kernels do not wait on one another).
dnb_status noalloc_after_launch(cudaStream_t s, const char *what) {
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DNB_ERR_CUDA, "launching %s failed: %s", what, cudaGetErrorString(e));
    if (sync_after_launch()) {
        e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) return fail(DNB_ERR_CUDA, "%s faulted: %s", what, cudaGetErrorString(e));
    }
    return DNB_OK;
}

}  // namespace
}  // namespace dnb

extern "C" dnb_status dnb_mean_noalloc(const float *x, int64_t batch, int64_t filters, int64_t spatial, float *out,
                                       dnb_stream stream) {
    using namespace dnb;
    const char *what = "mean_noalloc";
    if (batch < 0 || filters < 0 || spatial < 0) return fail(DNB_ERR_INVALID, "%s: negative size", what);
    if (filters == 0) return DNB_OK;
    if (!out || (batch * spatial > 0 && !x)) return fail(DNB_ERR_INVALID, "%s: null pointer", what);
    if (filters > 65535) return fail(DNB_ERR_UNSUPPORTED, "%s: more than 65535 channels", what);
    // the geometry dnb_mean uses (chan_reduce), so both produce the same partials
    Geometry g;
    g.batch = batch;
    g.filters = filters;
    g.spatial = spatial;
    g.per_channel = batch * spatial;
    g.vec = spatial % 4 == 0 && aligned16(x);
    g.chunk = kChunkElems;
    int64_t chunks = (g.per_channel + g.chunk - 1) / g.chunk;
    if (chunks < 1) chunks = 1;
    g.chunks = (int)chunks;
    g.fast = g.per_channel < (1ll << 32);
    if (spatial > 0) {
        g.fs = FastDiv((uint32_t)(g.fast ? spatial : 1));
        g.fs4 = FastDiv((uint32_t)(g.fast && g.vec ? spatial / 4 : 1));
    }
    if (filters * chunks > kNoAllocScratchFloats)
        return fail(DNB_ERR_UNSUPPORTED,
                    "%s: needs %lld partial sums (filters * ceil(batch*spatial/%lld)); the fixed scratch holds %lld",
                    what, (long long)(filters * chunks), (long long)kChunkElems, (long long)kNoAllocScratchFloats);
    float *partial = nullptr;
    DNB_TRY(noalloc_scratch(&partial));
    const cudaStream_t s = as_stream(stream);
    if (g.per_channel > 0) {
        k_chan_partial<TermSum, false><<<dim3((unsigned)chunks, (unsigned)filters), kThreads, 0, s>>>(g, x, nullptr,
                                                                                                   nullptr, partial);
    } else {
        // the previous call's partials are still there: clear the slots this call reads
        DNB_CUDA(cudaMemsetAsync(partial, 0, sizeof(float) * (size_t)(filters * chunks), s));
    }
    DNB_TRY(noalloc_after_launch(s, what));
    const float scale = 1.0f / (float)(batch * spatial);  // blas.zig:107
    const unsigned warps_per_block = 8;
    const unsigned blocks = (unsigned)((filters + warps_per_block - 1) / warps_per_block);
    k_chan_close<<<blocks, 32 * warps_per_block, 0, s>>>(filters, g.chunks, partial, Close::Mean, scale, nullptr, out);
    return noalloc_after_launch(s, what);
}
