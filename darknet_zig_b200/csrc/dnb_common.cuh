// Shared declarations for libdnb200: host-side error plumbing, per-device and per-stream
// state, and the device helpers every kernel file uses.
//
// All kernels are compiled with --fmad=false: the reference's CPU ops run in Zig's strict
// float mode, where a*b+c is two roundings. Where the reference fuses (blas.axpy in
// optimized float mode, blas.zig:21-24) the kernels call __fmaf_rn explicitly.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "dnb200.h"

namespace dnb {

// --------------------------------------------------------------------------------------
// host side
// --------------------------------------------------------------------------------------

// Records `detail` as this thread's last error and returns `s`.
dnb_status fail(dnb_status s, const char *fmt, ...);
dnb_status cuda_fail(cudaError_t e, const char *what, const char *file, int line);

#define DNB_CUDA(call)                                                                 \
    do {                                                                               \
        cudaError_t dnb_e_ = (call);                                                   \
        if (dnb_e_ != cudaSuccess) return ::dnb::cuda_fail(dnb_e_, #call, __FILE__, __LINE__); \
    } while (0)

#define DNB_TRY(expr)                     \
    do {                                  \
        dnb_status dnb_s_ = (expr);       \
        if (dnb_s_ != DNB_OK) return dnb_s_; \
    } while (0)

// Device-side error word bits (DeviceState::error_word).
enum : unsigned {
    DEVERR_WAIT_BARRIER = 1u,  // a CTA gave up waiting for the other CTAs of its grid
    DEVERR_WAIT_PEER = 4u,     // gave up waiting for another GPU
};

constexpr int kMaxDevices = 64;  // device ordinals the per-device state covers

struct DeviceState {
    int device = -1;
    int sm_count = 0;
    int max_smem_optin = 0;        // bytes of dynamic shared memory a CTA may opt into
    int smem_per_sm = 0;           // shared memory of one SM
    int smem_reserved = 0;         // shared memory the system reserves per CTA
    unsigned *error_word = nullptr;  // device: DEVERR_* bits, sticky until dnb_check_device_error
    unsigned *abort_flag = nullptr;  // device: set with the error word, makes other waiters give up
};

// Scratch owned by the library for one (device, stream) pair.
struct Workspace {
    cudaStream_t stream = nullptr;
    // persistent-kernel state: [0] = launch epoch, [1] = CTAs that finished the current launch;
    // [2] = blocks of the fused softmax + cross entropy that have left their row losses
    unsigned *sync = nullptr;
    size_t sync_words = 0;
    void *scratch = nullptr;  // per-channel partials of the multi-launch paths
    size_t scratch_bytes = 0;
    // the sweep's tagged per-CTA records (64-bit words), cleared when allocated or reset
    unsigned long long *recs = nullptr;
    size_t rec_words = 0;
};

constexpr size_t kSyncWords = 3;
constexpr size_t kSyncSoftmaxDone = 2;

// A sync-BN communicator as a kernel sees it (dnb_comm.cu): this rank, the ranks, and every
// rank's exchange buffer of tagged records, 64-bit words
// [2 parities][kMaxSweepGroups][world][pmax CTAs][2 segments][4].
constexpr int kMaxRanks = 8;
constexpr int kMaxSweepGroups = 64;
struct CommView {
    int rank = 0, world = 1;
    unsigned tag = 0;  // the call number (never 0): the records' tag; parity = tag & 1
    int pmax = 0;      // CTAs a group's records have room for
    int64_t cmax = 0;
    unsigned long long *rec[kMaxRanks] = {};
};
// The view of `comm` for its next fused call on the current device (advances its call number).
dnb_status comm_next(dnb_comm comm, CommView *out);

// The state of the current device, initialising it on first use.
dnb_status current_device(DeviceState **out);
// The workspace of (current device, stream) with at least `scratch_bytes` of scratch and
// `rec_words` record words.
dnb_status workspace(cudaStream_t stream, size_t scratch_bytes, Workspace **out, size_t rec_words = 0);
// Checks the launch that was just issued (and synchronises under sync-after-launch).
dnb_status after_launch(cudaStream_t stream, const char *what);
// Counts one device-side launch (kernel or memset) for dnb_launch_count; after_launch does it.
void note_launch();
// Spin limit for device-side waits, in nanoseconds.
unsigned long long wait_limit_ns();
// True under dnb_set_sync_after_launch(1).
bool sync_after_launch();

inline cudaStream_t as_stream(dnb_stream s) { return reinterpret_cast<cudaStream_t>(s); }
inline bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Grid size for a grid-stride loop over `items` work items.
inline unsigned grid_for(int64_t items, int threads, const DeviceState *ds, int per_sm = 8) {
    int64_t blocks = (items + threads - 1) / threads;
    int64_t cap = (int64_t)ds->sm_count * per_sm;
    if (blocks > cap) blocks = cap;
    if (blocks < 1) blocks = 1;
    return (unsigned)blocks;
}

// --------------------------------------------------------------------------------------
// device side
// --------------------------------------------------------------------------------------

// Unsigned division by a runtime-invariant divisor: q = mulhi(n, magic) >> shift, exact for
// every 32-bit n (Granlund & Montgomery, "Division by invariant integers using
// multiplication", PLDI 1994, with the 33-bit magic split into an add step).
struct FastDiv {
    uint32_t d = 1, magic = 0, shift = 0;
    FastDiv() = default;
    explicit FastDiv(uint32_t divisor) : d(divisor) {
        if (divisor == 1) { magic = 0; shift = 0; return; }
        uint32_t l = 0;
        while ((1ull << l) < divisor) ++l;  // l = ceil(log2 d)
        // magic = floor(2^32 * (2^l - d) / d) + 1
        magic = (uint32_t)(((1ull << 32) * ((1ull << l) - divisor)) / divisor + 1);
        shift = l;
    }
    __device__ __forceinline__ uint32_t div(uint32_t n) const {
        if (d == 1) return n;
        uint32_t t = __umulhi(n, magic);
        return (t + ((n - t) >> 1)) >> (shift - 1);
    }
    __device__ __forceinline__ void divmod(uint32_t n, uint32_t &q, uint32_t &r) const {
        q = div(n);
        r = n - q * d;
    }
};

__device__ __forceinline__ float4 ld4(const float *p) { return *reinterpret_cast<const float4 *>(p); }
__device__ __forceinline__ void st4(float *p, float4 v) { *reinterpret_cast<float4 *>(p) = v; }
// L2-only load (bypasses L1) for data another CTA will read again from L2.
__device__ __forceinline__ float4 ld4_l2(const float *p) { return __ldcg(reinterpret_cast<const float4 *>(p)); }
// Streaming (evict-first) variants for data touched exactly once.
__device__ __forceinline__ float4 ld4_stream(const float *p) { return __ldcs(reinterpret_cast<const float4 *>(p)); }
__device__ __forceinline__ void st4_stream(float *p, float4 v) { __stcs(reinterpret_cast<float4 *>(p), v); }

// ---- activations, darknet numbering (activations.zig:11-27) ----
// The arithmetic follows activations.zig:58-105 (the CPU twins), not the reference's
// device kernels: e.g. relu(x<0) is +0.0 (a select, activations.zig:63), tanh is
// (e-1)/(e+1) with e = exp(2x) (activations.zig:69-72).

// Zig folds 1.0507 * 1.6732 at comptime and rounds once to f32 (activations.zig:65,95).
#define DNB_SELU_SCALE_ALPHA ((float)(1.0507 * 1.6732))

__device__ __forceinline__ float act_fwd_any(float x, int a) {
    switch (a) {
    case DNB_ACT_LINEAR: return x;
    case DNB_ACT_LOGISTIC: return 1.0f / (1.0f + expf(-x));
    case DNB_ACT_LOGGY: return 2.0f / (1.0f + expf(-x)) - 1.0f;
    case DNB_ACT_RELU: return x > 0.0f ? x : 0.0f;
    case DNB_ACT_ELU: return x >= 0.0f ? x : expf(x) - 1.0f;
    case DNB_ACT_SELU: return x >= 0.0f ? 1.0507f * x : DNB_SELU_SCALE_ALPHA * (expf(x) - 1.0f);
    case DNB_ACT_RELIE: return x > 0.0f ? x : 0.01f * x;
    case DNB_ACT_RAMP: return (x > 0.0f ? x : 0.0f) + 0.1f * x;
    case DNB_ACT_LEAKY: return x > 0.0f ? x : 0.1f * x;
    case DNB_ACT_TANH: {
        float e = expf(2.0f * x);
        return (e - 1.0f) / (e + 1.0f);
    }
    case DNB_ACT_PLSE:
        if (x < -4.0f) return 0.01f * (x + 4.0f);
        if (x > 4.0f) return 0.01f * (x - 4.0f) + 1.0f;
        return 0.125f * x + 0.5f;
    case DNB_ACT_STAIR: {
        float n = floorf(x);
        long long ni = (long long)n;
        if (ni % 2 == 0) return floorf(x / 2.0f);
        return (x - n) + floorf(x / 2.0f);
    }
    case DNB_ACT_HARDTAN: {
        float lo = x < 1.0f ? x : 1.0f;
        return lo > -1.0f ? lo : -1.0f;
    }
    case DNB_ACT_LHTAN:
        if (x < 0.0f) return 0.001f * x;
        if (x > 1.0f) return 0.001f * (x - 1.0f) + 1.0f;
        return x;
    }
    return 0.0f;
}

__device__ __forceinline__ float act_grad_any(float y, int a) {
    switch (a) {
    case DNB_ACT_LINEAR: return 1.0f;
    case DNB_ACT_LOGISTIC: return (1.0f - y) * y;
    case DNB_ACT_LOGGY: {
        float t = (y + 1.0f) / 2.0f;
        return 2.0f * (1.0f - t) * t;
    }
    case DNB_ACT_RELU: return y > 0.0f ? 1.0f : 0.0f;
    case DNB_ACT_ELU: return y >= 0.0f ? 1.0f : y + 1.0f;
    case DNB_ACT_SELU: return y >= 0.0f ? 1.0507f : y + DNB_SELU_SCALE_ALPHA;
    case DNB_ACT_RELIE: return y > 0.0f ? 1.0f : 0.01f;
    case DNB_ACT_RAMP: return (y > 0.0f ? 1.0f : 0.0f) + 0.1f;
    case DNB_ACT_LEAKY: return y > 0.0f ? 1.0f : 0.1f;
    case DNB_ACT_TANH: return 1.0f - y * y;
    case DNB_ACT_PLSE: return (y < 0.0f || y > 1.0f) ? 0.01f : 0.125f;
    case DNB_ACT_STAIR: return floorf(y) == y ? 0.0f : 1.0f;
    case DNB_ACT_HARDTAN: return (y > -1.0f && y < 1.0f) ? 1.0f : 0.0f;
    case DNB_ACT_LHTAN: return (y > 0.0f && y < 1.0f) ? 1.0f : 0.001f;
    }
    return 0.0f;
}

// Compile-time activation: A >= 0 is a fixed code, A == -1 dispatches on the runtime code.
template <int A>
__device__ __forceinline__ float act_fwd(float x, int a) {
    if constexpr (A == DNB_ACT_LEAKY) return x > 0.0f ? x : 0.1f * x;
    else if constexpr (A == DNB_ACT_RELU) return x > 0.0f ? x : 0.0f;
    else if constexpr (A == DNB_ACT_LINEAR) return x;
    else if constexpr (A == DNB_ACT_LOGISTIC) return 1.0f / (1.0f + expf(-x));
    else return act_fwd_any(x, a);
}
template <int A>
__device__ __forceinline__ float act_grad(float y, int a) {
    if constexpr (A == DNB_ACT_LEAKY) return y > 0.0f ? 1.0f : 0.1f;
    else if constexpr (A == DNB_ACT_RELU) return y > 0.0f ? 1.0f : 0.0f;
    else if constexpr (A == DNB_ACT_LINEAR) return 1.0f;
    else if constexpr (A == DNB_ACT_LOGISTIC) return (1.0f - y) * y;
    else return act_grad_any(y, a);
}

// Calls f.template operator()<A>() with the activation code as a template argument for the
// four activations the fused kernels specialise, and A = -1 for the rest.
template <class F>
auto dispatch_act(int act, F &&f) {
    switch (act) {
    case DNB_ACT_LEAKY: return f.template operator()<DNB_ACT_LEAKY>();
    case DNB_ACT_RELU: return f.template operator()<DNB_ACT_RELU>();
    case DNB_ACT_LINEAR: return f.template operator()<DNB_ACT_LINEAR>();
    case DNB_ACT_LOGISTIC: return f.template operator()<DNB_ACT_LOGISTIC>();
    default: return f.template operator()<-1>();
    }
}

inline bool valid_act(int a) { return a >= 0 && a <= 13; }

// ---- warp / block reductions ----
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ double warp_sum(double v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Sum over the block; every thread gets the result. `red` holds >= 32 floats of shared
// memory; the call begins and ends with a __syncthreads().
template <int NT>
__device__ __forceinline__ float block_sum(float v, float *red) {
    static_assert(NT % 32 == 0 && NT <= 1024, "block size");
    constexpr int W = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = lane < W ? red[lane] : 0.0f;
    return warp_sum(t);
}

// Two sums at once (same contract as block_sum; `red` holds >= 64 floats).
template <int NT>
__device__ __forceinline__ float2 block_sum2(float a, float b, float *red) {
    constexpr int W = NT / 32;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    a = warp_sum(a);
    b = warp_sum(b);
    __syncthreads();
    if (lane == 0) {
        red[warp] = a;
        red[32 + warp] = b;
    }
    __syncthreads();
    float ta = lane < W ? red[lane] : 0.0f;
    float tb = lane < W ? red[32 + lane] : 0.0f;
    return make_float2(warp_sum(ta), warp_sum(tb));
}

// ---- bounded waits ----
__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned ld_volatile(const unsigned *p) {
    return *reinterpret_cast<const volatile unsigned *>(p);
}

}  // namespace dnb
