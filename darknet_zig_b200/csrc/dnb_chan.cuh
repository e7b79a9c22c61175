// Per-channel broadcast driver shared by the elementwise and batchnorm files: element e of
// an NCHW tensor belongs to channel (e / spatial) % filters, and each block stages the
// per-channel parameter records it needs in shared memory once.
#pragma once

#include "dnb_common.cuh"

namespace dnb {
namespace chan {

constexpr int kThreads = 256;
constexpr int kUnroll = 4;

// A float4 at e = 4*i spans one channel when S % 4 == 0 and at most two when S >= 4.
struct ChanMap {
    FastDiv fs, fc;  // divide by S, by C
    uint32_t S;
    bool same4;      // S % 4 == 0
    __device__ __forceinline__ uint32_t chan(uint32_t e) const {
        uint32_t p = fs.div(e);
        uint32_t q, c;
        fc.divmod(p, q, c);
        return c;
    }
    // channels of elements e..e+3 (e = 4*i; requires S >= 4)
    __device__ __forceinline__ void chan4(uint32_t e, uint32_t ch[4]) const {
        uint32_t p, r;
        fs.divmod(e, p, r);
        uint32_t q, c;
        fc.divmod(p, q, c);
        ch[0] = ch[1] = ch[2] = ch[3] = c;
        if (!same4 && r + 3 >= S) {
            const uint32_t c2 = (c + 1 == fc.d) ? 0 : c + 1;
#pragma unroll
            for (int k = 1; k < 4; ++k)
                if (r + k >= S) ch[k] = c2;
        }
    }
};

inline ChanMap make_chan_map(int64_t filters, int64_t spatial) {
    ChanMap m;
    m.fs = FastDiv((uint32_t)spatial);
    m.fc = FastDiv((uint32_t)filters);
    m.S = (uint32_t)spatial;
    m.same4 = (spatial % 4) == 0;
    return m;
}

// Shapes the 32-bit channel map covers; larger tensors use 64-bit division.
inline bool chan_map_ok(int64_t total, int64_t spatial) { return total < (1ll << 32) - 8 && spatial >= 4; }

// Broadcast op driver: P is a per-channel parameter record staged into shared memory
// once per block (param(c) builds it from the op's per-channel arrays).
template <class Op>
__global__ void __launch_bounds__(kThreads) k_chan(int64_t n, int64_t channels, int64_t spatial, ChanMap cm, bool fast,
                                                  Op op) {
    extern __shared__ __align__(16) unsigned char smem_raw[];
    using P = typename Op::P;
    P *tab = reinterpret_cast<P *>(smem_raw);
    for (int64_t c = threadIdx.x; c < channels; c += kThreads) tab[c] = op.param(c);
    __syncthreads();
    const int64_t n4 = (fast && op.vec) ? (n >> 2) : 0;
    const int64_t tile = (int64_t)kThreads * kUnroll;
    for (int64_t base = (int64_t)blockIdx.x * tile; base < n4; base += (int64_t)gridDim.x * tile) {
        typename Op::V v[kUnroll];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads + threadIdx.x;
            if (i < n4) v[u] = op.load(i);
        }
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
            const int64_t i = base + u * kThreads + threadIdx.x;
            if (i < n4) {
                uint32_t ch[4];
                cm.chan4((uint32_t)(4 * i), ch);
                op.store(i, v[u], tab[ch[0]], tab[ch[1]], tab[ch[2]], tab[ch[3]]);
            }
        }
    }
    const int64_t step = (int64_t)gridDim.x * kThreads;
    for (int64_t j = (n4 << 2) + (int64_t)blockIdx.x * kThreads + threadIdx.x; j < n; j += step) {
        const int64_t c = fast ? (int64_t)cm.chan((uint32_t)j) : (j / spatial) % channels;
        op.scalar(j, tab[c]);
    }
}

template <class Op>
dnb_status launch_chan(int64_t batch, int64_t filters, int64_t spatial, const Op &op, cudaStream_t stream,
                       const char *what) {
    if (batch < 0 || filters < 0 || spatial < 0) return fail(DNB_ERR_INVALID, "%s: negative size", what);
    const int64_t n = batch * filters * spatial;
    if (n == 0) return DNB_OK;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const size_t smem = sizeof(typename Op::P) * (size_t)filters;
    if (smem > (size_t)ds->max_smem_optin)
        return fail(DNB_ERR_UNSUPPORTED, "%s: %lld channels exceed the per-block parameter table", what,
                    (long long)filters);
    if (smem > 48 * 1024)
        DNB_CUDA(cudaFuncSetAttribute(k_chan<Op>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    const bool fast = chan_map_ok(n, spatial);
    const ChanMap cm = fast ? make_chan_map(filters, spatial) : ChanMap{};
    const int64_t items = (fast && op.vec) ? ((n >> 2) + kUnroll - 1) / kUnroll : n;
    k_chan<Op><<<grid_for(items, kThreads, ds), kThreads, smem, stream>>>(n, filters, spatial, cm, fast, op);
    return after_launch(stream, what);
}

}  // namespace chan
}  // namespace dnb
