// Device helpers shared by the two persistent batchnorm + activation kernels (the L2 sweep
// in dnb_bn.cu and the shared-memory-staged kernel in dnb_bn_stage.cu): the per-channel
// closing formulas, the tagged per-CTA records of the grid-wide exchange, the balanced
// partition of a channel group into CTA shares, and the host-side I/O bundle both launchers
// take.
//
// Per-element arithmetic follows the reference CPU code (blas.zig:137-204) operation by
// operation without fused roundings (--fmad=false), so given the same per-channel
// statistics the outputs are bit-identical to it.
#pragma once

#include <math.h>

#include "dnb_cdiv.cuh"
#include "dnb_chan.cuh"

namespace dnb {

// The tensors and per-channel vectors of one fused call. Forward: t0 = x, out = y (xnorm
// optional); backward: t0 = delta, t1 = x, t2 = y (optional), out = dx.
struct BnIO {
    const float *t0 = nullptr, *t1 = nullptr, *t2 = nullptr;
    float *out = nullptr, *xnorm = nullptr;
    const float *scales = nullptr, *biases = nullptr;
    float *mean = nullptr, *var = nullptr, *rmean = nullptr, *rvar = nullptr;
    const float *mean_in = nullptr, *var_in = nullptr;
    float *bias_upd = nullptr, *scale_upd = nullptr, *mean_delta = nullptr, *var_delta = nullptr;
};

// Launches the shared-memory-staged kernel (dnb_bn_stage.cu) when its plan takes the shape;
// *launched says whether it did. With a communicator view the statistics span every rank.
template <bool BWD, bool HASY>
dnb_status run_stage(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                     bool *launched, const char *what, const CommView *cv);
// DNB_BN_STAGE=0 turns the staged kernel off.
bool stage_disabled();
// Launches the cluster-per-channel kernel (dnb_bn_cluster.cu) when its plan takes the shape.
template <bool BWD, bool HASY>
dnb_status run_cluster(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                       bool *launched, const char *what, const CommView *cv);
// DNB_BN_CLUSTER=0 turns the cluster kernel off.
bool cluster_disabled();
// Launches the channel-per-CTA kernel for small channels (dnb_bn_small.cu) when a channel's
// inputs fit its shared memory; single GPU only.
template <bool BWD, bool HASY>
dnb_status run_small(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                     bool *launched, const char *what);
// DNB_BN_SMALL=0 turns the small-channel kernel off.
bool small_disabled();


namespace {

// ======================================================================================
// per-channel closing formulas shared by both paths
// ======================================================================================

// Forward: statistics -> outputs and the per-channel apply record.
// mean/var rounding: the reference computes sum*(1/n) and sum*(1/(n-1)) in f32
// (blas.zig:107,122); here the fp64 merge result is rounded once.
struct FwdClose {
    float m, var, inv;
};
__device__ __forceinline__ FwdClose fwd_close(double mean, double m2, double count) {
    FwdClose r;
    r.m = (float)mean;
    r.var = (float)(m2 / (count - 1.0));
    r.inv = 1.0f / (sqrtf(r.var) + 0.000001f);  // blas.zig:142
    return r;
}
// batchnorm.zig:140-143: scal(0.99) then axpy(1-0.99) with one fused rounding
__device__ __forceinline__ float rolling(float r, float stat) { return __fmaf_rn(1.0f - 0.99f, stat, r * 0.99f); }

struct BwdParam {
    float m, inv, g, b;       // forward normalisation (to recompute y) and scale/bias
    float inv2, vd, mdd, pad;  // normalize_delta terms: 1/sqrt(v+1e-5), variance_delta, mean_delta/denom
};

// Backward closing: s1 = sum(g), s2 = sum(g*(x-m)) over the whole (global) channel.
// bwd_params gives the apply parameters; bwd_write the per-channel outputs (the mean and
// variance deltas are p.mdd * denom's unrounded source md and p.vd, recomputed identically).
__device__ __forceinline__ BwdParam bwd_params(double s1, double s2, float m, float var, float gamma, float beta,
                                               float denom, float *md_out = nullptr) {
    BwdParam p;
    p.m = m;
    p.inv = 1.0f / (sqrtf(var) + 0.000001f);
    p.g = gamma;
    p.b = beta;
    p.inv2 = 1.0f / sqrtf(var + 0.00001f);                                               // blas.zig:195
    const float md = (float)((double)gamma * s1) * (-1.0f / sqrtf(var + 0.00001f));      // blas.zig:155
    const float vd = (float)((double)gamma * s2) * -0.5f * powf(var + 0.00001f, -1.5f);  // blas.zig:176
    p.vd = vd;
    p.mdd = md / denom;
    p.pad = 0.0f;
    if (md_out) *md_out = md;
    return p;
}
__device__ __forceinline__ void bwd_write(double s1, double s2, const BwdParam &p, float md, float *bias_upd,
                                          float *scale_upd, float *mean_delta, float *var_delta, int64_t c) {
    bias_upd[c] += (float)s1;                      // blas.zig:79
    scale_upd[c] += (float)(s2 * (double)p.inv);  // sum(g * x_norm), blas.zig:98
    mean_delta[c] = md;
    var_delta[c] = p.vd;
}
__device__ __forceinline__ BwdParam bwd_close(double s1, double s2, float m, float var, float gamma, float beta,
                                              float denom, float *bias_upd, float *scale_upd, float *mean_delta,
                                              float *var_delta, int64_t c, bool write) {
    float md;
    const BwdParam p = bwd_params(s1, s2, m, var, gamma, beta, denom, &md);
    if (write) bwd_write(s1, s2, p, md, bias_upd, scale_upd, mean_delta, var_delta, c);
    return p;
}

// y = act(((x - m) * inv) * gamma + beta): normalize, scaleBias, addBias, activate
template <int A>
__device__ __forceinline__ float bn_fwd1(float x, float m, float inv, float g, float b, int act) {
    return act_fwd<A>((x - m) * inv * g + b, act);
}
// g = delta * act'(y); y from the given output or recomputed from x
template <int A, bool HASY>
__device__ __forceinline__ float bn_grad1(float d, float x, float y, const BwdParam &p, int act) {
    const float yy = HASY ? y : bn_fwd1<A>(x, p.m, p.inv, p.g, p.b, act);
    return d * act_grad<A>(yy, act);
}
template <int A, bool HASY>
__device__ __forceinline__ float4 bn_grad4(float4 d, float4 x, float4 y, const BwdParam &p, int act) {
    return make_float4(bn_grad1<A, HASY>(d.x, x.x, y.x, p, act), bn_grad1<A, HASY>(d.y, x.y, y.y, p, act),
                       bn_grad1<A, HASY>(d.z, x.z, y.z, p, act), bn_grad1<A, HASY>(d.w, x.w, y.w, p, act));
}


// A record is 4 64-bit words, each (tag << 32 | a float's bits): naturally aligned 64-bit
// accesses are single-copy atomic, so a word read with this launch's tag carries this
// launch's value, and a record whose words all carry it is complete. No fence, counter or
// flag orders a record: the merger polls the records themselves.
__device__ __forceinline__ unsigned long long tag_word(float v, unsigned tag) {
    return ((unsigned long long)tag << 32) | __float_as_uint(v);
}
template <int NW>  // words that carry data: 3 (count, mean, M2) or 2 (two sums)
__device__ __forceinline__ void st_record(unsigned long long *p, float4 q, unsigned tag, bool sys) {
    const unsigned long long w0 = tag_word(q.x, tag), w1 = tag_word(q.y, tag);
    if (sys)
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
    else
        asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
    if constexpr (NW > 2) {
        const unsigned long long w2 = tag_word(q.z, tag), w3 = tag_word(0.0f, tag);
        if (sys)
            asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 2), "l"(w2), "l"(w3) : "memory");
        else
            asm volatile("st.relaxed.gpu.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 2), "l"(w2), "l"(w3) : "memory");
    }
}
// true once every data word of the record at p carries `tag`; q then holds its values
template <int NW>
__device__ __forceinline__ bool ld_record(const unsigned long long *p, unsigned tag, bool sys, float4 &q) {
    unsigned long long w0, w1, w2 = 0, w3 = 0;
    if (sys)
        asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
    else
        asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
    if constexpr (NW > 2) {
        if (sys)
            asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w2), "=l"(w3) : "l"(p + 2) : "memory");
        else
            asm volatile("ld.relaxed.gpu.global.v2.b64 {%0, %1}, [%2];" : "=l"(w2), "=l"(w3) : "l"(p + 2) : "memory");
    }
    q = make_float4(__uint_as_float((unsigned)w0), __uint_as_float((unsigned)w1), __uint_as_float((unsigned)w2), 0.0f);
    bool ok = (unsigned)(w0 >> 32) == tag && (unsigned)(w1 >> 32) == tag;
    if constexpr (NW > 2) ok = ok && (unsigned)(w2 >> 32) == tag;
    return ok;
}

// Share of CTA p of a role with `parts` CTAs in group g: units [t0, t1) of the group's T,
// in at most two channel segments (the plan keeps shares no longer than a channel).
struct Share {
    uint32_t c0, T, t0, t1, bnd;  // bnd: first unit of the second segment
    int cfirst, nseg;
};
template <class Args>
__device__ __forceinline__ Share share_of(const Args &a, int g, int p, const FastDiv &parts) {
    Share s;
    s.c0 = (uint32_t)g * (uint32_t)a.cg;
    s.T = g == a.G - 1 ? a.T_last : a.T_full;
    s.t0 = parts.div((uint32_t)p * s.T);
    s.t1 = parts.div((uint32_t)(p + 1) * s.T);
    s.cfirst = (int)a.f_nk.div(s.t0);
    s.bnd = (uint32_t)(s.cfirst + 1) * (uint32_t)a.NK;
    s.nseg = s.t1 <= s.t0 ? 0 : (s.t1 <= s.bnd ? 1 : 2);
    return s;
}
// The CTA (of a role with `parts` CTAs) that owns unit t of group g.
template <class Args>
__device__ __forceinline__ int owner_of(const Args &a, int g, uint32_t t, int parts) {
    const FastDiv &fd = g == a.G - 1 ? a.f_tlast : a.f_tfull;
    return (int)fd.div((t + 1) * (uint32_t)parts - 1);
}

template <class Args>
__device__ __forceinline__ float div_denom(float v, const Args &a) {
    return div_const(v, a.cdiv);
}
// dx = (g*gamma)*inv2 + vd*2*(x-m)/denom + md/denom (blas.zig:200 on delta*scales), the division
// by the element count done by the launch's ConstDiv
template <class Args>
__device__ __forceinline__ float bn_dx_p(float gval, float x, const BwdParam &p, const Args &a) {
    return (gval * p.g) * p.inv2 + div_denom(p.vd * 2.0f * (x - p.m), a) + p.mdd;
}
// the same for four elements (g and x of a float4)
template <class Args>
__device__ __forceinline__ float4 bn_dx4_p(float4 g, float4 x, const BwdParam &p, const Args &a) {
    const float k = p.vd * 2.0f;
    const float4 q = div4_const(make_float4(k * (x.x - p.m), k * (x.y - p.m), k * (x.z - p.m), k * (x.w - p.m)), a.cdiv);
    return make_float4((g.x * p.g) * p.inv2 + q.x + p.mdd, (g.y * p.g) * p.inv2 + q.y + p.mdd,
                       (g.z * p.g) * p.inv2 + q.z + p.mdd, (g.w * p.g) * p.inv2 + q.w + p.mdd);
}

// Chan et al.'s combination of two (count, mean, M2) summaries.
__device__ __forceinline__ void chan_merge(float &n, float &m, float &q, float nb, float mb, float qb) {
    const float nn = n + nb;
    if (nn > 0.0f) {
        const float d = mb - m;
        const float f = nb / nn;
        m = m + d * f;
        q = q + qb + d * d * n * f;
        n = nn;
    }
}

// Per-thread running moments of one segment, shifted by the first value the thread saw.
struct Moments {
    float shift = 0.0f, s1 = 0.0f, s2 = 0.0f, n = 0.0f;
    __device__ __forceinline__ void add4(float4 v) {
        if (n == 0.0f) shift = v.x;
        const float d0 = v.x - shift, d1 = v.y - shift, d2 = v.z - shift, d3 = v.w - shift;
        s1 += (d0 + d1) + (d2 + d3);
        s2 += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
        n += 4.0f;
    }
    __device__ __forceinline__ void add1(float v) {
        if (n == 0.0f) shift = v;
        const float d = v - shift;
        s1 += d;
        s2 += d * d;
        n += 1.0f;
    }
    // warp-wide (count, mean, M2), valid in every lane
    __device__ __forceinline__ float4 warp_summary() const {
        float m = n > 0.0f ? shift + s1 / n : 0.0f;
        float q = n > 0.0f ? s2 - s1 * (s1 / n) : 0.0f;
        if (q < 0.0f) q = 0.0f;
        float c = n;
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float cb = __shfl_xor_sync(0xffffffffu, c, o);
            const float mb = __shfl_xor_sync(0xffffffffu, m, o);
            const float qb = __shfl_xor_sync(0xffffffffu, q, o);
            chan_merge(c, m, q, cb, mb, qb);
        }
        return make_float4(c, m, q, 0.0f);
    }
};


__device__ __forceinline__ uint64_t l2_evict_last() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, %1;" : "=l"(p) : "f"(1.0f));
    return p;
}
__device__ __forceinline__ uint64_t l2_evict_first() {
    uint64_t p;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, %1;" : "=l"(p) : "f"(1.0f));
    return p;
}
__device__ __forceinline__ float4 ld4_hint(const float *p, uint64_t pol) {
    float4 v;
    asm volatile("ld.global.L1::no_allocate.L2::cache_hint.v4.f32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ void st4_hint(float *p, float4 v, uint64_t pol) {
    asm volatile("st.global.L1::no_allocate.L2::cache_hint.v4.f32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w), "l"(pol)
                 : "memory");
}


// ---- mbarrier and bulk-copy primitives (PTX) ----
__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t *bar, unsigned count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, unsigned bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}
// try_wait with a suspend-time hint: the thread may sleep up to `ns` nanoseconds in the
// instruction until the phase completes (no polling loop of its own in the meantime)
__device__ __forceinline__ bool mbar_try_wait_ns(uint64_t *bar, unsigned parity, unsigned ns) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity), "r"(ns)
        : "memory");
    return ok;
}
__device__ __forceinline__ bool mbar_test(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// global -> shared bulk copy of `bytes` (multiple of 16, both addresses 16-byte aligned),
// completing on `bar`; evict-first in L2 (every input byte is read once)
__device__ __forceinline__ void bulk_load(void *dst, const void *src, unsigned bytes, uint64_t *bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar)), "l"(pol)
        : "memory");
}

// shared -> global bulk copy (both addresses 16-byte aligned, bytes a multiple of 16), in the
// issuing thread's current bulk group
__device__ __forceinline__ void bulk_store(void *dst, const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_addr(src)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// until at most N of this thread's bulk groups still read shared memory
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// until all of this thread's bulk groups are complete (their writes performed)
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// this thread's shared-memory writes, ordered before later bulk copies that read them
__device__ __forceinline__ void fence_proxy_async() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// bring `bytes` at src (16-byte aligned, a multiple of 16) into L2
__device__ __forceinline__ void prefetch_l2(const void *src, unsigned bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- thread-block cluster primitives (PTX) ----
// the address of the same shared-memory location in CTA `rank` of this cluster
__device__ __forceinline__ uint32_t cluster_map(const void *p, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(p)), "r"(rank));
    return r;
}
__device__ __forceinline__ void st_cluster_f64x2(uint32_t addr, double a, double b) {
    asm volatile("st.shared::cluster.v2.f64 [%0], {%1, %2};" ::"r"(addr), "d"(a), "d"(b) : "memory");
}
// arrive on an mbarrier of another CTA of the cluster, releasing this thread's earlier writes
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(addr) : "memory");
}
// mbar_test with cluster-scope acquire: also sees what other CTAs of the cluster released
__device__ __forceinline__ bool mbar_test_cluster(uint64_t *bar, unsigned parity) {
    unsigned ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// every thread of every CTA of the cluster (aligned: whole warps)
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}

inline int env_int(const char *name, int dflt, int lo, int hi) {
    const char *e = getenv(name);
    int v = e ? atoi(e) : dflt;
    return v < lo ? lo : (v > hi ? hi : v);
}

}  // namespace
}  // namespace dnb
