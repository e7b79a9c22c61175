// Fused batchnorm + activation, training forward and backward, for small channels: one CTA
// per channel, the whole channel in shared memory.
//
// Late layers of darknet's classifiers have small planes (7 x 7, 13 x 13, 14 x 14): a
// channel of a batch of 64 is a few tens of KB. The persistent kernels then spend their time
// on per-unit and per-group overheads, and the generic path on its four launches. Here a CTA
// loads its channel's N planes (every input tensor) into shared memory with coalesced loads,
// accumulating the statistics as it goes, reduces them over the block in fp64 in a fixed
// order, closes them into the apply parameters, and writes the outputs from shared memory.
// CTAs never wait for one another, so many channels are in flight on every SM; each input
// byte crosses HBM once and each output byte once. Single GPU only (sync-BN channels need
// the other ranks' statistics and go to the persistent kernels).
//
// Reference sequence this replaces: batchnorm.zig:129-174 with the activation of
// convolutional.zig:269/280.
#include <atomic>

#include "dnb_bn.cuh"

namespace dnb {
namespace {

constexpr int kSmThreads = 256;
constexpr int kSmWarps = kSmThreads / 32;
constexpr size_t kSmMaxBytes = 96 * 1024;  // a channel's inputs must fit this

struct SmArgs {
    int64_t C, S;
    int N;
    FastDiv fs;     // divide by S
    int vec;        // S % 4 == 0 and aligned tensors: float4 access
    float denom;
    ConstDiv cdiv;  // division by denom, per element
    BnIO io;
    int act;
};

// Block-wide fp64 totals of two per-thread float sums, added warp by warp in warp order
// (every thread gets the same totals).
__device__ __forceinline__ double2 block_totals(float a, float b, double2 *red) {
    a = warp_sum(a);
    b = warp_sum(b);
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (lane == 0) red[warp] = make_double2((double)a, (double)b);
    __syncthreads();
    double2 t = make_double2(0.0, 0.0);
    for (int w = 0; w < kSmWarps; ++w) {
        t.x += red[w].x;
        t.y += red[w].y;
    }
    __syncthreads();
    return t;
}

template <bool BWD, int A, bool HASY>
__global__ void __launch_bounds__(kSmThreads) k_bn_small(SmArgs a) {
    constexpr int NT = BWD ? (HASY ? 3 : 2) : 1;
    extern __shared__ __align__(16) float ch[];  // [NT][N * S]
    __shared__ double2 red[kSmWarps];
    __shared__ float prm[8];
    const int64_t NS = (int64_t)a.N * a.S;
    const float *src[3] = {a.io.t0, a.io.t1, a.io.t2};
    for (int64_t c = blockIdx.x; c < a.C; c += gridDim.x) {
        float s1 = 0.0f, s2 = 0.0f;
        float K = 0.0f;
        BwdParam fp;
        if (BWD) {
            const float m = a.io.mean_in[c], v = a.io.var_in[c];
            fp.m = m;
            fp.inv = 1.0f / (sqrtf(v) + 0.000001f);  // the forward's normalisation, batchnorm.zig:142
            fp.g = a.io.scales[c];
            fp.b = a.io.biases[c];
        } else {
            K = a.io.t0[c * a.S];  // shift: the channel's first element
        }
        // load every input plane of the channel, accumulating the statistics
        if (a.vec) {
            const int64_t n4 = NS >> 2;
            const uint32_t s4 = (uint32_t)(a.S >> 2);
            for (int64_t e = threadIdx.x; e < n4; e += kSmThreads) {
                const uint32_t n = (uint32_t)e / s4, r = (uint32_t)e - n * s4;
                const int64_t g = ((int64_t)n * a.C + c) * a.S + 4 * (int64_t)r;
                float4 v[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    v[t] = ld4_stream(src[t] + g);
                    reinterpret_cast<float4 *>(ch + t * NS)[e] = v[t];
                }
                if constexpr (!BWD) {
                    const float d0 = v[0].x - K, d1 = v[0].y - K, d2 = v[0].z - K, d3 = v[0].w - K;
                    s1 += (d0 + d1) + (d2 + d3);
                    s2 += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
                } else {
                    const float4 yy = HASY ? v[NT - 1] : v[1];
                    const float g0 = bn_grad1<A, HASY>(v[0].x, v[1].x, yy.x, fp, a.act);
                    const float g1 = bn_grad1<A, HASY>(v[0].y, v[1].y, yy.y, fp, a.act);
                    const float g2 = bn_grad1<A, HASY>(v[0].z, v[1].z, yy.z, fp, a.act);
                    const float g3 = bn_grad1<A, HASY>(v[0].w, v[1].w, yy.w, fp, a.act);
                    s1 += (g0 + g1) + (g2 + g3);
                    s2 += (g0 * (v[1].x - fp.m) + g1 * (v[1].y - fp.m)) + (g2 * (v[1].z - fp.m) + g3 * (v[1].w - fp.m));
                }
            }
        } else {
            for (int64_t e = threadIdx.x; e < NS; e += kSmThreads) {
                uint32_t n, r;
                a.fs.divmod((uint32_t)e, n, r);
                const int64_t g = ((int64_t)n * a.C + c) * a.S + r;
                float v[NT];
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                    v[t] = src[t][g];
                    ch[t * NS + e] = v[t];
                }
                if constexpr (!BWD) {
                    const float d = v[0] - K;
                    s1 += d;
                    s2 += d * d;
                } else {
                    const float gv = bn_grad1<A, HASY>(v[0], v[1], HASY ? v[NT - 1] : 0.0f, fp, a.act);
                    s1 += gv;
                    s2 += gv * (v[1] - fp.m);
                }
            }
        }
        const double2 tot = block_totals(s1, s2, red);
        if (threadIdx.x == 0) {
            if constexpr (!BWD) {
                const double n = (double)NS;
                const double mean = (double)K + tot.x / n;
                double m2 = tot.y - tot.x * (tot.x / n);
                if (m2 < 0.0) m2 = 0.0;
                const FwdClose f = fwd_close(mean, m2, n);
                prm[0] = f.m;
                prm[1] = f.inv;
                prm[2] = a.io.scales[c];
                prm[3] = a.io.biases[c];
                a.io.mean[c] = f.m;
                a.io.var[c] = f.var;
                a.io.rmean[c] = rolling(a.io.rmean[c], f.m);
                a.io.rvar[c] = rolling(a.io.rvar[c], f.var);
            } else {
                float md;
                const BwdParam p =
                    bwd_params(tot.x, tot.y, a.io.mean_in[c], a.io.var_in[c], fp.g, fp.b, a.denom, &md);
                *reinterpret_cast<BwdParam *>(prm) = p;
                bwd_write(tot.x, tot.y, p, md, a.io.bias_upd, a.io.scale_upd, a.io.mean_delta, a.io.var_delta, c);
            }
        }
        __syncthreads();
        // the outputs from shared memory
        if constexpr (!BWD) {
            const float m = prm[0], inv = prm[1], g = prm[2], b = prm[3];
            if (a.vec) {
                const int64_t n4 = NS >> 2;
                const uint32_t s4 = (uint32_t)(a.S >> 2);
                for (int64_t e = threadIdx.x; e < n4; e += kSmThreads) {
                    const uint32_t n = (uint32_t)e / s4, r = (uint32_t)e - n * s4;
                    const int64_t o = ((int64_t)n * a.C + c) * a.S + 4 * (int64_t)r;
                    const float4 v = reinterpret_cast<const float4 *>(ch)[e];
                    if (a.io.xnorm)
                        st4(a.io.xnorm + o, make_float4((v.x - m) * inv, (v.y - m) * inv, (v.z - m) * inv,
                                                        (v.w - m) * inv));
                    st4_stream(a.io.out + o, make_float4(bn_fwd1<A>(v.x, m, inv, g, b, a.act),
                                                         bn_fwd1<A>(v.y, m, inv, g, b, a.act),
                                                         bn_fwd1<A>(v.z, m, inv, g, b, a.act),
                                                         bn_fwd1<A>(v.w, m, inv, g, b, a.act)));
                }
            } else {
                for (int64_t e = threadIdx.x; e < NS; e += kSmThreads) {
                    uint32_t n, r;
                    a.fs.divmod((uint32_t)e, n, r);
                    const int64_t o = ((int64_t)n * a.C + c) * a.S + r;
                    const float v = ch[e];
                    if (a.io.xnorm) a.io.xnorm[o] = (v - m) * inv;
                    a.io.out[o] = bn_fwd1<A>(v, m, inv, g, b, a.act);
                }
            }
        } else {
            const BwdParam p = *reinterpret_cast<const BwdParam *>(prm);
            if (a.vec) {
                const int64_t n4 = NS >> 2;
                const uint32_t s4 = (uint32_t)(a.S >> 2);
                for (int64_t e = threadIdx.x; e < n4; e += kSmThreads) {
                    const uint32_t n = (uint32_t)e / s4, r = (uint32_t)e - n * s4;
                    const int64_t o = ((int64_t)n * a.C + c) * a.S + 4 * (int64_t)r;
                    const float4 d = reinterpret_cast<const float4 *>(ch)[e];
                    const float4 xv = reinterpret_cast<const float4 *>(ch + NS)[e];
                    const float4 yy = HASY ? reinterpret_cast<const float4 *>(ch + 2 * NS)[e] : xv;
                    st4_stream(a.io.out + o, bn_dx4_p(bn_grad4<A, HASY>(d, xv, yy, p, a.act), xv, p, a));
                }
            } else {
                for (int64_t e = threadIdx.x; e < NS; e += kSmThreads) {
                    uint32_t n, r;
                    a.fs.divmod((uint32_t)e, n, r);
                    const int64_t o = ((int64_t)n * a.C + c) * a.S + r;
                    const float xv = ch[NS + e];
                    const float gv = bn_grad1<A, HASY>(ch[e], xv, HASY ? ch[2 * NS + e] : 0.0f, p, a.act);
                    a.io.out[o] = bn_dx_p(gv, xv, p, a);
                }
            }
        }
        __syncthreads();  // the channel's shared memory is read before the next channel's loads
    }
}

}  // namespace

bool small_disabled() {
    const char *e = getenv("DNB_BN_SMALL");
    return e && e[0] == '0';
}

template <bool BWD, bool HASY>
dnb_status run_small(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                     bool *launched, const char *what) {
    *launched = false;
    constexpr int nt = BWD ? (HASY ? 3 : 2) : 1;
    if (batch <= 0 || filters <= 0 || spatial <= 0) return DNB_OK;
    const int64_t NS = batch * spatial;
    const size_t smem = (size_t)nt * NS * sizeof(float);
    if (smem > kSmMaxBytes || NS >= (1ll << 31)) return DNB_OK;
    if ((uint64_t)batch * (uint64_t)filters * (uint64_t)spatial >= (1ull << 40)) return DNB_OK;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    const void *ts[4] = {io.t0, io.t1, io.t2, io.out};
    bool al = aligned16(io.out) && (!io.xnorm || aligned16(io.xnorm));
    for (int t = 0; t < nt; ++t) al = al && aligned16(ts[t]);
    SmArgs a{};
    a.C = filters;
    a.S = spatial;
    a.N = (int)batch;
    a.fs = FastDiv((uint32_t)spatial);
    a.vec = al && spatial % 4 == 0;
    a.denom = (float)(batch * spatial);
    a.cdiv = const_div(a.denom);
    a.io = io;
    a.act = act;
    return dispatch_act(act, [&]<int A>() -> dnb_status {
        auto kern = k_bn_small<BWD, A, HASY>;
        if (smem > 48 * 1024) {
            static std::atomic<int> set[kMaxDevices];
            if (!set[ds->device].load(std::memory_order_relaxed)) {
                DNB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmMaxBytes));
                set[ds->device].store(1, std::memory_order_relaxed);
            }
        }
        int occ = 0;
        DNB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kSmThreads, smem));
        if (occ < 1) return DNB_OK;
        const int64_t cap = (int64_t)ds->sm_count * occ;
        const unsigned grid = (unsigned)(filters < cap ? filters : cap);
        kern<<<grid, kSmThreads, smem, stream>>>(a);
        *launched = true;
        return after_launch(stream, what);
    });
}

template dnb_status run_small<false, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                            const char *);
template dnb_status run_small<true, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                           const char *);
template dnb_status run_small<true, true>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                          const char *);

}  // namespace dnb
