// Fused batchnorm + activation, training forward and backward: one thread-block cluster per
// channel at a time.
//
// The per-channel statistics must be complete before any output element of the channel can
// be written, so every element is used twice. Here a cluster of Q CTAs (one per SM) owns
// whole channels: clusters take channels k, k + nc, k + 2 nc, ... and each CTA of a cluster
// holds 1/Q of the channel's units (U consecutive floats of one image plane) in a ring of
// shared-memory slots. Per CTA:
//
//   producer warp   streams the CTA's units of channel after channel into the ring with TMA
//                   bulk copies (cp.async.bulk global -> shared, one per unit and tensor,
//                   completion on a per-slot mbarrier, no multicast), one unit per lane, as
//                   slots come free; it also prefetches the channel after next into L2;
//   stats warps     reduce each unit once it lands: forward sum(x - K) and sum((x - K)^2)
//                   about a shift K common to the whole channel (its first element), backward
//                   sum(g) and sum(g * (x - mean)), g = delta * act'(y);
//   exchange warp   adds the warps' partials in fp64, stores the CTA's partial into every
//                   CTA of the cluster (distributed shared memory) and arrives on their
//                   barriers, then adds the cluster's Q partials in rank order -- every CTA
//                   gets bit-identical totals -- and hands the channel's apply parameters to
//                   the output warps; with a communicator, the cluster's first CTA combines
//                   the cluster totals of every rank over NVLink first;
//   apply warps     write the outputs over the unit's slot and send them out with one TMA bulk
//                   copy per unit, then free the slot for the producer.
//
// Every byte crosses HBM once each way, clusters never wait for one another (on one GPU),
// and a channel's exchange is a shared-memory round trip inside the cluster, overlapped
// with the loads of the channels behind it. Waits are bounded (%globaltimer); a CTA that
// gives up sets the device error word and the abort flag, its warps stop, its copies are
// drained, and the cluster meets once more before it exits so that no CTA leaves while
// another may still write into its shared memory.
//
// Reference sequence this replaces: batchnorm.zig:129-174 with the activation of
// convolutional.zig:269/280.
#include <stdio.h>
#include <stdlib.h>

#include <atomic>

#include "dnb_bn.cuh"

namespace dnb {
namespace {

constexpr int kCStats = 4;                           // statistics warps
constexpr int kCApply = 8;                           // output warps
constexpr int kCWarps = 1 + kCStats + kCApply + 1;   // + producer, exchange
constexpr int kCThreads = 32 * kCWarps;
constexpr int kCWarpStats0 = 1;
constexpr int kCWarpApply0 = kCWarpStats0 + kCStats;
constexpr int kCWarpExch = kCWarpApply0 + kCApply;
constexpr int kCRing = 8;             // channel-state buffers; fewer channels are ever in flight
constexpr int kCMaxSlots = 256;
constexpr int kCMaxUnitFloats = 2048;  // preferred unit size: at most 8 KB per tensor
constexpr int kCMaxQ = 16;
constexpr int kCMaxChannels = 256;     // channels of one cluster the prologue tables hold
constexpr int kCStaticSmemReserve = 1024;

struct CArgs {
    int64_t C, S;
    int N, K, U, NK;
    int Q, nc;                 // CTAs per cluster, clusters
    int R, SU, slot_floats, vec, bulk_out;
    int pf_from;               // first channel (of a cluster's sequence) prefetched into L2
    FastDiv f_k;
    float denom;               // normalize_delta's denominator (all ranks' elements)
    ConstDiv cdiv;             // division by denom, per element
    double count;              // elements behind a channel's statistics (all ranks)
    BnIO io;
    int act;
    unsigned *err, *abort_flag;
    unsigned long long wait_ns;
    // sync-BN: the cluster's first CTA stores the cluster's totals of channel c into every
    // rank's buffer (a record of 6 tagged 64-bit words at ((xpar * xcmax + c) * world + rank)
    // * 8) and reads every rank's from its own
    int xon, world, rank, xpar;
    unsigned xtag;
    int64_t xcmax;
    unsigned long long *xrec[kMaxRanks];
};

template <bool BWD, int A, bool HASY>
struct Clu {
    static constexpr int NT = BWD ? (HASY ? 3 : 2) : 1;

    struct Smem {
        float *ring;      // [R][slot_floats]
        uint64_t *full;   // [R] the slot's unit has landed
        uint64_t *empty;  // [R] the slot's unit has been written out
        // channel-state buffer b = j % kCRing for the cluster's j-th channel; each barrier
        // completes one phase per channel that uses the buffer (parity (j / kCRing) & 1)
        float2 *wpart;    // [DB][kCStats] per statistics warp
        double2 *xpart;   // [DB][kCMaxQ] the cluster CTAs' partials, written by each CTA
        double2 *gtot;    // [DB] with a communicator: the totals over every rank
        double *gshift;   // [DB] ... and the shift they are taken about (rank 0's)
        float *ptab;      // [DB][8] apply parameters
        uint64_t *sbar;   // [DB] every statistics warp has left its partial
        uint64_t *xbar;   // [DB] every CTA of the cluster has stored its partial here
        uint64_t *gbar;   // [DB] the cross-rank totals are in gtot
        uint64_t *rbar;   // [DB] the apply parameters are in ptab
        uint64_t *abar;   // [DB] every output warp is done with the channel
        // per channel of this cluster [kCMaxChannels], loaded once in the prologue:
        float4 *ctab;     // (gamma, beta, shift K) or (mean, var, gamma, beta)
        float4 *stab;     // backward: the forward's (mean, inv, gamma, beta)
        float2 *otab;     // prior (rolling mean, rolling var) or (bias_updates, scale_updates)
        uint64_t *tbar;   // the tables are loaded
        int *stop;        // set when any wait of this CTA gave up
    };
    static size_t ctrl_bytes(int R) {
        return (size_t)R * 16 +
               (size_t)kCRing * (kCStats * sizeof(float2) + kCMaxQ * sizeof(double2) + sizeof(double2) +
                                 sizeof(double) + 8 * sizeof(float) + 5 * sizeof(uint64_t)) +
               (size_t)kCMaxChannels * (2 * sizeof(float4) + sizeof(float2)) + 64;
    }
    static size_t smem_bytes(int R, int slot_floats) { return (size_t)R * slot_floats * sizeof(float) + ctrl_bytes(R); }
    __device__ static Smem carve(const CArgs &a, unsigned char *raw) {
        Smem s;
        size_t o = 0;
        s.ring = reinterpret_cast<float *>(raw);
        o += (size_t)a.R * a.slot_floats * sizeof(float);
        s.full = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)a.R * 8;
        s.empty = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)a.R * 8;
        s.xpart = reinterpret_cast<double2 *>(raw + o);
        o += (size_t)kCRing * kCMaxQ * sizeof(double2);
        s.gtot = reinterpret_cast<double2 *>(raw + o);
        o += (size_t)kCRing * sizeof(double2);
        s.gshift = reinterpret_cast<double *>(raw + o);
        o += (size_t)kCRing * sizeof(double);
        s.wpart = reinterpret_cast<float2 *>(raw + o);
        o += (size_t)kCRing * kCStats * sizeof(float2);
        s.ptab = reinterpret_cast<float *>(raw + o);
        o += (size_t)kCRing * 8 * sizeof(float);
        s.sbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kCRing * sizeof(uint64_t);
        s.xbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kCRing * sizeof(uint64_t);
        s.gbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kCRing * sizeof(uint64_t);
        s.rbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kCRing * sizeof(uint64_t);
        s.abar = reinterpret_cast<uint64_t *>(raw + o);
        o += kCRing * sizeof(uint64_t);
        s.ctab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)kCMaxChannels * sizeof(float4);
        s.stab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)kCMaxChannels * sizeof(float4);
        s.otab = reinterpret_cast<float2 *>(raw + o);
        o += (size_t)kCMaxChannels * sizeof(float2);
        s.tbar = reinterpret_cast<uint64_t *>(raw + o);
        o += sizeof(uint64_t);
        s.stop = reinterpret_cast<int *>(raw + o);
        return s;
    }

    // ---- geometry ----
    // channels of cluster k: k, k + nc, ...; this many
    __device__ static int n_channels(const CArgs &a, int k) { return (int)((a.C - k + a.nc - 1) / a.nc); }
    // units [lo, hi) of a channel belong to CTA r of the cluster
    __device__ static uint32_t unit_lo(const CArgs &a, int r) { return (uint32_t)((int64_t)r * a.NK / a.Q); }
    // element offset of unit u of channel c (the plan keeps offsets below 2^32)
    __device__ static uint32_t unit_offset(const CArgs &a, int64_t c, uint32_t u) {
        uint32_t n, kk;
        a.f_k.divmod(u, n, kk);
        return ((n * (uint32_t)a.C + (uint32_t)c) * (uint32_t)a.S) + kk * (uint32_t)a.U;
    }

    // ---- waits (all bounded, warp-uniform) ----
    __device__ static void give_up(const CArgs &a, const Smem &s, unsigned bit) {
        atomicOr(a.err, bit);
        atomicExch(a.abort_flag, 1u);
        *reinterpret_cast<volatile int *>(s.stop) = 1;
    }
    __device__ static bool stopped(const Smem &s) { return *reinterpret_cast<const volatile int *>(s.stop) != 0; }
    // lane 0's verdict after a failed test: 1 to stop waiting (this CTA stopped, another CTA or
    // kernel gave up, or the wait ran out)
    __device__ static int quit_now(const CArgs &a, const Smem &s, unsigned long long deadline, unsigned &polls,
                                   unsigned bit) {
        if (stopped(s)) return 1;
        if ((++polls & 15u) == 0 && ld_volatile(a.abort_flag)) {
            *reinterpret_cast<volatile int *>(s.stop) = 1;
            return 1;
        }
        if (global_ns() > deadline) {
            give_up(a, s, bit);
            return 1;
        }
        return 0;
    }
    template <bool CLUSTER>
    __device__ static bool wait_bar(const CArgs &a, const Smem &s, uint64_t *bar, unsigned parity) {
        auto test = [&]() { return CLUSTER ? mbar_test_cluster(bar, parity) : mbar_test(bar, parity); };
        if (__all_sync(0xffffffffu, test())) return true;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        unsigned polls = 0;
        for (;;) {
            if (__all_sync(0xffffffffu, test())) return true;
            int quit = 0;
            if ((threadIdx.x & 31) == 0) quit = quit_now(a, s, deadline, polls, DEVERR_WAIT_BARRIER);
            if (__shfl_sync(0xffffffffu, quit, 0)) return false;
            __nanosleep(64);
        }
    }
    __device__ static bool wait_chan(const CArgs &a, const Smem &s, uint64_t *bars, int j) {
        return wait_bar<false>(a, s, &bars[j % kCRing], (unsigned)(j / kCRing) & 1u);
    }
    __device__ static void arrive_chan(uint64_t *bars, int j) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&bars[j % kCRing]);
        __syncwarp();
    }

    // ---- prologue (every warp but the producer): the per-channel tables ----
    __device__ static void load_tables(const CArgs &a, const Smem &s, int k, int r) {
        const int J = n_channels(a, k);
        for (int j = (int)threadIdx.x - 32; j < J; j += kCThreads - 32) {
            const int64_t c = (int64_t)k + (int64_t)j * a.nc;
            if (BWD) {
                const float m = a.io.mean_in[c], v = a.io.var_in[c], gm = a.io.scales[c], bt = a.io.biases[c];
                s.ctab[j] = make_float4(m, v, gm, bt);
                // the forward's normalisation (batchnorm.zig:142), to recompute y from x
                s.stab[j] = make_float4(m, 1.0f / (sqrtf(v) + 0.000001f), gm, bt);
                if (r == 0) s.otab[j] = make_float2(a.io.bias_upd[c], a.io.scale_upd[c]);
            } else {
                // shift: the channel's first element (plane 0), the same in every CTA of the
                // cluster; with a communicator it is this rank's, and the totals of the ranks
                // are re-centred on rank 0's shift before they are added
                s.ctab[j] = make_float4(a.io.scales[c], a.io.biases[c], a.io.t0[c * a.S], 0.0f);
                if (r == 0) s.otab[j] = make_float2(a.io.rmean[c], a.io.rvar[c]);
            }
        }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(s.tbar);
        __syncwarp();
    }

    // ---- producer warp ----
    // Units are numbered in the CTA's order of channels and units; unit i lives in slot i % R
    // and is that slot's (i / R)-th occupant. A channel's share of units is at most R, so a
    // unit waits only for slots of earlier channels, and the lanes of one batch (at most
    // min(32, R) units of one channel) never wait for one another.
    __device__ static void producer(const CArgs &a, const Smem &s, int k, int r) {
        const int lane = threadIdx.x & 31;
        const uint64_t pol = l2_evict_first();
        const uint32_t width = a.R < 32 ? (uint32_t)a.R : 32u;
        const uint32_t lo = unit_lo(a, r), n_units = unit_lo(a, r + 1) - lo;
        const int J = n_channels(a, k);
        uint32_t i0 = 0, issued = 0;
        bool ok = true;
        for (int j = 0; j < J && ok; ++j) {
            // channel j reuses the state buffer of channel j - kCRing
            if (j >= kCRing && !wait_chan(a, s, s.abar, j - kCRing)) break;
            const int64_t c = (int64_t)k + (int64_t)j * a.nc;
            for (uint32_t base = 0; base < n_units && ok; base += width) {
                const uint32_t u = base + (uint32_t)lane;
                const bool has = (uint32_t)lane < width && u < n_units;
                const uint32_t i = i0 + u, slot = i % (uint32_t)a.R, use = i / (uint32_t)a.R;
                bool free_ = !has || use == 0 || mbar_test(&s.empty[slot], (use - 1) & 1u);
                if (!__all_sync(0xffffffffu, free_)) {
                    const unsigned long long deadline = global_ns() + a.wait_ns;
                    unsigned polls = 0;
                    for (;;) {
                        free_ = free_ || mbar_test(&s.empty[slot], (use - 1) & 1u);
                        if (__all_sync(0xffffffffu, free_)) break;
                        int quit = 0;
                        if (lane == 0) quit = quit_now(a, s, deadline, polls, DEVERR_WAIT_BARRIER);
                        if (__shfl_sync(0xffffffffu, quit, 0)) {
                            ok = false;
                            break;
                        }
                        __nanosleep(64);
                    }
                    if (!ok) break;  // no unit of this batch was issued
                }
                if (has) {
                    const uint32_t off = unit_offset(a, c, lo + u);
                    const uint32_t start = a.vec ? off : (off & ~3u);
                    const uint32_t len = a.vec ? (uint32_t)a.U : ((off - start + (uint32_t)a.U + 3u) & ~3u);
                    float *dst = s.ring + (size_t)slot * a.slot_floats;
                    mbar_arrive_expect_tx(&s.full[slot], (unsigned)(NT * len * 4));
                    bulk_load(dst, a.io.t0 + start, len * 4, &s.full[slot], pol);
                    if (NT > 1) bulk_load(dst + a.SU, a.io.t1 + start, len * 4, &s.full[slot], pol);
                    if (NT > 2) bulk_load(dst + 2 * a.SU, a.io.t2 + start, len * 4, &s.full[slot], pol);
                }
                __syncwarp();
                issued = i0 + (base + width < n_units ? base + width : n_units);
            }
            i0 += n_units;
            // the share of the channel after next into L2: its loads are issued once slots
            // come free and then come from L2 (the channels that fit the ring at the start are
            // loaded at once and need no prefetch)
            const int q = j + 2;
            if (ok && q < J && q >= a.pf_from) {
                const int64_t cq = (int64_t)k + (int64_t)q * a.nc;
                for (uint32_t u = lane; u < n_units; u += 32) {
                    const uint32_t off = unit_offset(a, cq, lo + u);
                    const uint32_t start = a.vec ? off : (off & ~3u);
                    const uint32_t len = a.vec ? (uint32_t)a.U : ((off - start + (uint32_t)a.U + 3u) & ~3u);
                    prefetch_l2(a.io.t0 + start, len * 4);
                    if (NT > 1) prefetch_l2(a.io.t1 + start, len * 4);
                    if (NT > 2) prefetch_l2(a.io.t2 + start, len * 4);
                }
                __syncwarp();
            }
        }
        // every copy issued into this CTA's shared memory lands before the CTA may exit: the
        // slots' current occupants, the last R units issued
        const uint32_t first = issued > (uint32_t)a.R ? issued - (uint32_t)a.R : 0u;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        for (uint32_t q = first + (uint32_t)lane; q < issued; q += 32) {
            const uint32_t slot = q % (uint32_t)a.R;
            while (!mbar_test(&s.full[slot], (q / (uint32_t)a.R) & 1u) && global_ns() < deadline) __nanosleep(64);
        }
        __syncwarp();
    }

    // ---- statistics warps ----
    __device__ static void stats(const CArgs &a, const Smem &s, int k, int r, int ws) {
        const int lane = threadIdx.x & 31;
        if (!wait_bar<false>(a, s, s.tbar, 0)) return;  // the shift (forward) or stab (backward)
        const uint32_t lo = unit_lo(a, r), n_units = unit_lo(a, r + 1) - lo;
        const int J = n_channels(a, k);
        uint32_t i0 = 0;
        for (int j = 0; j < J; ++j) {
            // a warp without units would otherwise overwrite wpart of channel j - kCRing
            // before the exchange warp has read it
            if (j >= kCRing && !wait_chan(a, s, s.rbar, j - kCRing)) return;
            // every statistics warp is done with channel j - 1, so every unit of the earlier
            // channels has landed: the previous occupant of each slot this warp waits on
            // below. Without it a warp running a channel ahead could test a slot's `full`
            // barrier while the phase of the slot's previous unit is still open, and a parity
            // wait one phase early succeeds at once (stale data in the sums).
            if (j >= 1 && !wait_chan(a, s, s.sbar, j - 1)) return;
            const int64_t c = (int64_t)k + (int64_t)j * a.nc;
            float s1 = 0.0f, s2 = 0.0f;
            if constexpr (!BWD) {
                const float K = s.ctab[j].z;
                for (uint32_t u = ws; u < n_units; u += kCStats) {
                    const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                    if (!wait_bar<false>(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) return;
                    const float *src = s.ring + (size_t)slot * a.slot_floats;
                    if (a.vec) {
                        const float4 *v4 = reinterpret_cast<const float4 *>(src);
                        const int n4 = a.U >> 2;
#pragma unroll 4
                        for (int q = lane; q < n4; q += 32) {
                            const float4 v = v4[q];
                            const float d0 = v.x - K, d1 = v.y - K, d2 = v.z - K, d3 = v.w - K;
                            s1 += (d0 + d1) + (d2 + d3);
                            s2 += (d0 * d0 + d1 * d1) + (d2 * d2 + d3 * d3);
                        }
                    } else {
                        const uint32_t o = unit_offset(a, c, lo + u) & 3u;
                        for (int q = lane; q < a.U; q += 32) {
                            const float d = src[o + q] - K;
                            s1 += d;
                            s2 += d * d;
                        }
                    }
                }
            } else {
                const float4 fp = s.stab[j];
                BwdParam p;
                p.m = fp.x;
                p.inv = fp.y;
                p.g = fp.z;
                p.b = fp.w;
                for (uint32_t u = ws; u < n_units; u += kCStats) {
                    const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                    if (!wait_bar<false>(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) return;
                    const float *src = s.ring + (size_t)slot * a.slot_floats;
                    if (a.vec) {
                        const float4 *d4 = reinterpret_cast<const float4 *>(src);
                        const float4 *x4 = reinterpret_cast<const float4 *>(src + a.SU);
                        const float4 *y4 = reinterpret_cast<const float4 *>(src + 2 * a.SU);
                        const int n4 = a.U >> 2;
#pragma unroll 2
                        for (int q = lane; q < n4; q += 32) {
                            const float4 d = d4[q], xv = x4[q];
                            const float4 yy = HASY ? y4[q] : xv;
                            const float g0 = bn_grad1<A, HASY>(d.x, xv.x, yy.x, p, a.act);
                            const float g1 = bn_grad1<A, HASY>(d.y, xv.y, yy.y, p, a.act);
                            const float g2 = bn_grad1<A, HASY>(d.z, xv.z, yy.z, p, a.act);
                            const float g3 = bn_grad1<A, HASY>(d.w, xv.w, yy.w, p, a.act);
                            s1 += (g0 + g1) + (g2 + g3);
                            s2 += (g0 * (xv.x - p.m) + g1 * (xv.y - p.m)) + (g2 * (xv.z - p.m) + g3 * (xv.w - p.m));
                        }
                    } else {
                        const uint32_t o = unit_offset(a, c, lo + u) & 3u;
                        for (int q = lane; q < a.U; q += 32) {
                            const float xv = src[a.SU + o + q];
                            const float gv =
                                bn_grad1<A, HASY>(src[o + q], xv, HASY ? src[2 * a.SU + o + q] : 0.0f, p, a.act);
                            s1 += gv;
                            s2 += gv * (xv - p.m);
                        }
                    }
                }
            }
            const float t1 = warp_sum(s1), t2 = warp_sum(s2);
            if (lane == 0) s.wpart[(j % kCRing) * kCStats + ws] = make_float2(t1, t2);
            arrive_chan(s.sbar, j);
            i0 += n_units;
        }
    }

    // ---- exchange warp ----
    __device__ static size_t xword(const CArgs &a, int64_t c, int q) {
        return (((size_t)a.xpar * (size_t)a.xcmax + (size_t)c) * a.world + q) * 8;
    }
    // A cross-rank record: the two fp64 totals as four tagged 32-bit halves and the fp32
    // shift, every 64-bit word (tag << 32 | 32 data bits), stored and read as aligned 128-bit
    // pairs; complete once all six words carry this call's tag (the words of one record may
    // land in any order).
    __device__ static void st_xrec(unsigned long long *p, double t1, double t2, float shift, unsigned tag) {
        const unsigned long long hi = (unsigned long long)tag << 32;
        const unsigned long long b1 = __double_as_longlong(t1), b2 = __double_as_longlong(t2);
        const unsigned long long w0 = hi | (b1 & 0xffffffffull), w1 = hi | (b1 >> 32);
        const unsigned long long w2 = hi | (b2 & 0xffffffffull), w3 = hi | (b2 >> 32);
        const unsigned long long w4 = hi | __float_as_uint(shift), w5 = hi;
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p), "l"(w0), "l"(w1) : "memory");
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 2), "l"(w2), "l"(w3) : "memory");
        asm volatile("st.relaxed.sys.global.v2.b64 [%0], {%1, %2};" ::"l"(p + 4), "l"(w4), "l"(w5) : "memory");
    }
    __device__ static bool ld_xrec(const unsigned long long *p, unsigned tag, double &t1, double &t2, float &shift) {
        unsigned long long w0, w1, w2, w3, w4, w5;
        asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w0), "=l"(w1) : "l"(p) : "memory");
        asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w2), "=l"(w3) : "l"(p + 2) : "memory");
        asm volatile("ld.relaxed.sys.global.v2.b64 {%0, %1}, [%2];" : "=l"(w4), "=l"(w5) : "l"(p + 4) : "memory");
        const bool ok = (unsigned)(w0 >> 32) == tag && (unsigned)(w1 >> 32) == tag && (unsigned)(w2 >> 32) == tag &&
                        (unsigned)(w3 >> 32) == tag && (unsigned)(w4 >> 32) == tag && (unsigned)(w5 >> 32) == tag;
        t1 = __longlong_as_double((long long)((w1 << 32) | (w0 & 0xffffffffull)));
        t2 = __longlong_as_double((long long)((w3 << 32) | (w2 & 0xffffffffull)));
        shift = __uint_as_float((unsigned)w4);
        return ok;
    }
    // the leader's cross-rank step: this cluster's totals to every rank, every rank's back,
    // added in rank order (identical on every rank), then into gtot of every CTA of the cluster
    __device__ static bool exchange_ranks(const CArgs &a, const Smem &s, int64_t c, int b, double t1, double t2,
                                          double shift) {
        const int lane = threadIdx.x & 31;
        // a rank's record: its totals and (forward) the shift they are about
        if (lane < a.world) st_xrec(a.xrec[lane] + xword(a, c, a.rank), t1, t2, (float)shift, a.xtag);
        double r1 = 0.0, r2 = 0.0;
        float rk = 0.0f;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        unsigned polls = 0;
        for (;;) {
            const bool done = lane >= a.world || ld_xrec(a.xrec[a.rank] + xword(a, c, lane), a.xtag, r1, r2, rk);
            if (__all_sync(0xffffffffu, done)) break;
            int quit = 0;
            if (lane == 0) quit = quit_now(a, s, deadline, polls, DEVERR_WAIT_PEER);
            if (__shfl_sync(0xffffffffu, quit, 0)) return false;
            __nanosleep(64);
        }
        // in rank order: the totals about rank 0's shift k0 (forward), so that every rank adds
        // the same numbers in the same order
        const double k0 = (double)__shfl_sync(0xffffffffu, rk, 0);
        double g1 = 0.0, g2 = 0.0;
        const double n_rank = a.count / a.world;
        for (int q = 0; q < a.world; ++q) {
            const double q1 = __shfl_sync(0xffffffffu, r1, q);
            const double q2 = __shfl_sync(0xffffffffu, r2, q);
            if (BWD) {
                g1 += q1;
                g2 += q2;
            } else {
                // sum (x - k0) = q1 + n dk; sum (x - k0)^2 = q2 + 2 dk q1 + n dk^2, dk = kq - k0
                const double dk = (double)__shfl_sync(0xffffffffu, rk, q) - k0;
                g1 += q1 + n_rank * dk;
                g2 += q2 + 2.0 * dk * q1 + n_rank * dk * dk;
            }
        }
        if (lane < a.Q) {
            st_cluster_f64x2(cluster_map(&s.gtot[b], lane), g1, g2);
            const uint32_t ks = cluster_map(&s.gshift[b], lane);
            asm volatile("st.shared::cluster.f64 [%0], %1;" ::"r"(ks), "d"(k0) : "memory");
            mbar_arrive_cluster(cluster_map(&s.gbar[b], lane));
        }
        __syncwarp();
        return true;
    }

    __device__ static void exchange(const CArgs &a, const Smem &s, int k, int r) {
        const int lane = threadIdx.x & 31;
        if (!wait_bar<false>(a, s, s.tbar, 0)) return;
        const int J = n_channels(a, k);
        for (int j = 0; j < J; ++j) {
            const int b = j % kCRing;
            const unsigned ph = (unsigned)(j / kCRing) & 1u;
            const int64_t c = (int64_t)k + (int64_t)j * a.nc;
            if (!wait_bar<false>(a, s, &s.sbar[b], ph)) return;
            // this CTA's partial (fp64, warps in order) into every CTA of the cluster
            double p1 = 0.0, p2 = 0.0;
            for (int w = 0; w < kCStats; ++w) {
                const float2 v = s.wpart[b * kCStats + w];
                p1 += (double)v.x;
                p2 += (double)v.y;
            }
            if (lane < a.Q) {
                st_cluster_f64x2(cluster_map(&s.xpart[b * kCMaxQ + r], lane), p1, p2);
                mbar_arrive_cluster(cluster_map(&s.xbar[b], lane));
            }
            __syncwarp();
            if (!wait_bar<true>(a, s, &s.xbar[b], ph)) return;
            double t1 = 0.0, t2 = 0.0;
            for (int q = 0; q < a.Q; ++q) {
                const double2 v = s.xpart[b * kCMaxQ + q];
                t1 += v.x;
                t2 += v.y;
            }
            const float4 ci = s.ctab[j];
            double shift = BWD ? 0.0 : (double)ci.z;  // this channel's shift, the same in the cluster
            if (a.xon) {
                if (r == 0 && !exchange_ranks(a, s, c, b, t1, t2, shift)) {
                    if (lane == 0) *reinterpret_cast<volatile int *>(s.stop) = 1;
                    return;
                }
                if (!wait_bar<true>(a, s, &s.gbar[b], ph)) return;
                // the totals of every rank, about rank 0's shift: the same on every rank
                const double2 g = s.gtot[b];
                t1 = g.x;
                t2 = g.y;
                shift = s.gshift[b];
            }
            float md = 0.0f;
            FwdClose f;
            BwdParam p;
            if (lane == 0) {
                float *out = s.ptab + b * 8;
                if constexpr (!BWD) {
                    const double n = a.count;
                    const double mean = shift + t1 / n;
                    double m2 = t2 - t1 * (t1 / n);
                    if (m2 < 0.0) m2 = 0.0;
                    f = fwd_close(mean, m2, n);
                    *reinterpret_cast<float4 *>(out) = make_float4(f.m, f.inv, ci.x, ci.y);
                } else {
                    p = bwd_params(t1, t2, ci.x, ci.y, ci.z, ci.w, a.denom, &md);
                    *reinterpret_cast<BwdParam *>(out) = p;
                }
            }
            arrive_chan(s.rbar, j);
            // the per-channel outputs, by the cluster's first CTA
            if (r == 0 && lane == 0) {
                const float2 prior = s.otab[j];
                if constexpr (!BWD) {
                    a.io.mean[c] = f.m;
                    a.io.var[c] = f.var;
                    a.io.rmean[c] = rolling(prior.x, f.m);
                    a.io.rvar[c] = rolling(prior.y, f.var);
                } else {
                    a.io.bias_upd[c] = prior.x + (float)t1;  // blas.zig:79
                    a.io.scale_upd[c] = prior.y + (float)(t2 * (double)p.inv);  // blas.zig:98
                    a.io.mean_delta[c] = md;
                    a.io.var_delta[c] = p.vd;
                }
            }
            __syncwarp();
        }
    }

    // ---- output warps: outputs over the slot, one bulk copy out per unit ----
    __device__ static void apply(const CArgs &a, const Smem &s, int k, int r, int wa) {
        const int lane = threadIdx.x & 31;
        const uint32_t lo = unit_lo(a, r), n_units = unit_lo(a, r + 1) - lo;
        const int J = n_channels(a, k);
        uint32_t i0 = 0;
        int held = -1;  // lane 0: the slot whose bulk copy may still read it
        for (int j = 0; j < J; ++j) {
            const int b = j % kCRing;
            const int64_t c = (int64_t)k + (int64_t)j * a.nc;
            // every output warp waits for the channel's parameters, also one without units:
            // its arrival on abar below must not count towards an earlier channel's phase
            if (!wait_chan(a, s, s.rbar, j)) break;
            bool ok = true;
            for (uint32_t u = wa; u < n_units; u += kCApply) {
                const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                if (!wait_bar<false>(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) {
                    ok = false;
                    break;
                }
                const float *pt = s.ptab + b * 8;
                const uint32_t off = unit_offset(a, c, lo + u);
                float *src = s.ring + (size_t)slot * a.slot_floats;
                if constexpr (!BWD) {
                    const float4 p = *reinterpret_cast<const float4 *>(pt);
                    if (a.bulk_out) {
                        float4 *v4 = reinterpret_cast<float4 *>(src);
                        const int n4 = a.U >> 2;
#pragma unroll 4
                        for (int q = lane; q < n4; q += 32) {
                            const float4 v = v4[q];
                            v4[q] = make_float4(bn_fwd1<A>(v.x, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.y, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.z, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.w, p.x, p.y, p.z, p.w, a.act));
                        }
                    } else if (a.vec) {
                        const float4 *v4 = reinterpret_cast<const float4 *>(src);
                        const int n4 = a.U >> 2;
#pragma unroll 4
                        for (int q = lane; q < n4; q += 32) {
                            const float4 v = v4[q];
                            if (a.io.xnorm)
                                st4(a.io.xnorm + off + 4 * q, make_float4((v.x - p.x) * p.y, (v.y - p.x) * p.y,
                                                                          (v.z - p.x) * p.y, (v.w - p.x) * p.y));
                            st4(a.io.out + off + 4 * q, make_float4(bn_fwd1<A>(v.x, p.x, p.y, p.z, p.w, a.act),
                                                                    bn_fwd1<A>(v.y, p.x, p.y, p.z, p.w, a.act),
                                                                    bn_fwd1<A>(v.z, p.x, p.y, p.z, p.w, a.act),
                                                                    bn_fwd1<A>(v.w, p.x, p.y, p.z, p.w, a.act)));
                        }
                    } else {
                        const uint32_t o = off & 3u;
                        for (int q = lane; q < a.U; q += 32) {
                            const float v = src[o + q];
                            if (a.io.xnorm) a.io.xnorm[off + q] = (v - p.x) * p.y;
                            a.io.out[off + q] = bn_fwd1<A>(v, p.x, p.y, p.z, p.w, a.act);
                        }
                    }
                } else {
                    const BwdParam p = *reinterpret_cast<const BwdParam *>(pt);
                    if (a.vec) {
                        float4 *d4 = reinterpret_cast<float4 *>(src);
                        const float4 *x4 = reinterpret_cast<const float4 *>(src + a.SU);
                        const float4 *y4 = reinterpret_cast<const float4 *>(src + 2 * a.SU);
                        const int n4 = a.U >> 2;
#pragma unroll 2
                        for (int q = lane; q < n4; q += 32) {
                            const float4 d = d4[q], xv = x4[q];
                            const float4 yy = HASY ? y4[q] : xv;
                            const float4 o4 = bn_dx4_p(bn_grad4<A, HASY>(d, xv, yy, p, a.act), xv, p, a);
                            if (a.bulk_out)
                                d4[q] = o4;  // over delta, element by element
                            else
                                st4(a.io.out + off + 4 * q, o4);
                        }
                    } else {
                        const uint32_t o = off & 3u;
                        for (int q = lane; q < a.U; q += 32) {
                            const float xv = src[a.SU + o + q];
                            const float gv =
                                bn_grad1<A, HASY>(src[o + q], xv, HASY ? src[2 * a.SU + o + q] : 0.0f, p, a.act);
                            a.io.out[off + q] = bn_dx_p(gv, xv, p, a);
                        }
                    }
                }
                if (a.bulk_out) {
                    fence_proxy_async();  // the lanes' shared-memory writes, before the bulk copy reads them
                    __syncwarp();
                    if (lane == 0) {
                        bulk_store(a.io.out + off, src, (unsigned)a.U * 4u);
                        bulk_commit();
                        if (held >= 0) {
                            bulk_wait_read<1>();  // the previous unit's copy has read its slot
                            mbar_arrive(&s.empty[held]);
                        }
                        held = (int)slot;
                    }
                } else {
                    __syncwarp();
                    if (lane == 0) mbar_arrive(&s.empty[slot]);
                }
                __syncwarp();
            }
            if (lane == 0 && held >= 0) {
                bulk_wait_read<0>();
                mbar_arrive(&s.empty[held]);
                held = -1;
            }
            __syncwarp();
            if (!ok) break;
            arrive_chan(s.abar, j);
            i0 += n_units;
        }
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
};

template <bool BWD, int A, bool HASY>
__global__ void __launch_bounds__(kCThreads, 1) k_bn_cluster(CArgs a) {
    using K = Clu<BWD, A, HASY>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const typename K::Smem s = K::carve(a, smem_raw);
    const int r = (int)cluster_rank();
    const int k = (int)cluster_index();
    if (threadIdx.x == 0) {
        *s.stop = 0;
        mbar_init(s.tbar, kCWarps - 1);
    }
    if (threadIdx.x < kCRing) {
        mbar_init(&s.sbar[threadIdx.x], kCStats);
        mbar_init(&s.xbar[threadIdx.x], (unsigned)a.Q);
        mbar_init(&s.gbar[threadIdx.x], 1);
        mbar_init(&s.rbar[threadIdx.x], 1);
        mbar_init(&s.abar[threadIdx.x], kCApply);
    }
    for (int i = threadIdx.x; i < a.R; i += kCThreads) {
        mbar_init(&s.full[i], 1);
        mbar_init(&s.empty[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    // every CTA's barriers are initialised before any CTA of the cluster arrives on them
    cluster_sync_all();
    const int warp = threadIdx.x >> 5;
    if (warp != 0) K::load_tables(a, s, k, r);
    if (warp == 0) {
        K::producer(a, s, k, r);
    } else if (warp < kCWarpApply0) {
        K::stats(a, s, k, r, warp - kCWarpStats0);
    } else if (warp < kCWarpExch) {
        K::apply(a, s, k, r, warp - kCWarpApply0);
    } else {
        K::exchange(a, s, k, r);
    }
    // no CTA leaves while another CTA of the cluster may still write into its shared memory
    cluster_sync_all();
}

struct CPlan {
    bool ok = false;
    int K = 0, U = 0, SU = 0, R = 0, Q = 0, nc = 0, vec = 0, pf_from = 0;
    size_t smem = 0;
};

}  // namespace

bool cluster_disabled() {
    const char *e = getenv("DNB_BN_CLUSTER");
    return e && e[0] == '0';
}

template <bool BWD, bool HASY>
dnb_status run_cluster(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                       bool *launched, const char *what, const CommView *cv) {
    *launched = false;
    constexpr int nt = BWD ? (HASY ? 3 : 2) : 1;
    if (batch <= 0 || filters <= 0 || spatial <= 0) return DNB_OK;
    if ((uint64_t)batch * (uint64_t)filters * (uint64_t)spatial >= (1ull << 32) - 8) return DNB_OK;
    const void *ins[3] = {io.t0, io.t1, io.t2};
    for (int q = 0; q < nt; ++q)
        if (!aligned16(ins[q])) return DNB_OK;
    if (!aligned16(io.out) || (io.xnorm && !aligned16(io.xnorm))) return DNB_OK;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    using KS = Clu<BWD, DNB_ACT_LEAKY, HASY>;
    CPlan pl;
    pl.vec = spatial % 4 == 0;
    if (pl.vec) {
        int64_t kk = 0;
        for (int64_t q = 1; q <= spatial / 4; ++q)
            if (spatial % q == 0 && (spatial / q) % 4 == 0 && spatial / q <= kCMaxUnitFloats) {
                kk = q;
                break;
            }
        if (kk == 0) kk = 1;
        pl.K = (int)kk;
        pl.U = (int)(spatial / kk);
        pl.SU = pl.U;
    } else {
        // the aligned span of a plane may reach 3 floats past the tensor's end: only inside
        // the tensor when its element count is a multiple of 4
        if ((batch * filters * spatial) % 4 != 0) return DNB_OK;
        pl.K = 1;
        pl.U = (int)spatial;
        pl.SU = (int)((spatial + 6) & ~(int64_t)3);
    }
    const int dyn_max = ds->max_smem_optin - kCStaticSmemReserve;
    for (int R = kCMaxSlots; R >= 1; --R)
        if (KS::smem_bytes(R, nt * pl.SU) <= (size_t)dyn_max) {
            pl.R = R;
            break;
        }
    if (pl.R < 2) return DNB_OK;
    const int64_t NK = batch * pl.K;
    return dispatch_act(act, [&]<int A>() -> dnb_status {
        auto kern = k_bn_cluster<BWD, A, HASY>;
        // per device: the opt-in shared memory and the most clusters of each size that fit
        // (cached as 1 + count; sizes 1..16)
        static std::atomic<int> fits[kMaxDevices][5];
        static std::atomic<int> attr_done[kMaxDevices];
        if (!attr_done[ds->device].load(std::memory_order_relaxed)) {
            DNB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max));
            // 16-CTA clusters are beyond the portable limit of 8; a device that cannot hold them
            // reports no room for them below
            if (cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess)
                (void)cudaGetLastError();
            attr_done[ds->device].store(1, std::memory_order_relaxed);
        }
        // The cluster size Q: first by channels in flight (ring slots / a CTA's units per
        // channel: three or more, else two, else one), then by SMs in use (within 10 % counts
        // as equal), then the smaller Q (more clusters, finer channel granularity).
        int best_q = 0, best_nc = 0, best_tier = -1, best_sms = 0;
        for (int qi = 0; qi < 5; ++qi) {
            const int Q = 1 << qi;
            const int64_t m = (NK + Q - 1) / Q;  // units per CTA per channel
            if (m > pl.R) continue;
            int f1 = fits[ds->device][qi].load(std::memory_order_relaxed);
            if (f1 == 0) {
                cudaLaunchConfig_t cfg = {};
                cfg.gridDim = dim3((unsigned)Q);
                cfg.blockDim = dim3(kCThreads);
                cfg.dynamicSmemBytes = (size_t)dyn_max;
                cudaLaunchAttribute at[1];
                at[0].id = cudaLaunchAttributeClusterDimension;
                at[0].val.clusterDim.x = (unsigned)Q;
                at[0].val.clusterDim.y = 1;
                at[0].val.clusterDim.z = 1;
                cfg.attrs = at;
                cfg.numAttrs = 1;
                int n = 0;
                if (cudaOccupancyMaxActiveClusters(&n, kern, &cfg) != cudaSuccess) {
                    (void)cudaGetLastError();
                    n = 0;
                }
                f1 = n + 1;
                fits[ds->device][qi].store(f1, std::memory_order_relaxed);
            }
            const int ncmax = f1 - 1;
            if (ncmax < 1) continue;
            int64_t nc = ncmax < filters ? ncmax : filters;
            const int64_t rounds = (filters + nc - 1) / nc;
            nc = (filters + rounds - 1) / rounds;  // as few clusters as keep the same rounds
            const int64_t d = pl.R / m;
            const int tier = d >= 3 ? 2 : (d >= 2 ? 1 : 0);
            const int sms = (int)nc * Q;
            bool better;
            if (tier != best_tier)
                better = tier > best_tier;
            else if (sms * 10 > best_sms * 11 || best_sms * 10 > sms * 11)
                better = sms > best_sms;
            else
                better = false;  // equal within 10 %: keep the smaller Q found first
            if (better) {
                best_q = Q;
                best_nc = (int)nc;
                best_tier = tier;
                best_sms = sms;
            }
        }
        if (best_q == 0) return DNB_OK;
        const int J = (int)((filters + best_nc - 1) / best_nc);
        if (J > kCMaxChannels) return DNB_OK;
        pl.Q = best_q;
        pl.nc = best_nc;
        pl.pf_from = (int)(pl.R / ((NK + best_q - 1) / best_q));
        if (cv) {
            // the records ([2 parities][cmax channels][world][8 words]) must fit the exchange
            // buffer ([2][kMaxSweepGroups][world][pmax][8 words])
            if (filters > cv->cmax || cv->cmax > (int64_t)kMaxSweepGroups * cv->pmax) return DNB_OK;
        }
        if (const char *e = getenv("DNB_BN_PLAN_LOG"); e && e[0] == '1')
            fprintf(stderr, "dnb cluster plan: %s [%lld,%lld,%lld] K=%d U=%d R=%d Q=%d nc=%d units/CTA/channel=%lld\n",
                    what, (long long)batch, (long long)filters, (long long)spatial, pl.K, pl.U, pl.R, pl.Q, pl.nc,
                    (long long)((NK + pl.Q - 1) / pl.Q));
        CArgs a{};
        a.C = filters;
        a.S = spatial;
        a.N = (int)batch;
        a.K = pl.K;
        a.U = pl.U;
        a.NK = (int)NK;
        a.Q = pl.Q;
        a.nc = pl.nc;
        a.R = pl.R;
        a.SU = pl.SU;
        a.slot_floats = nt * pl.SU;
        a.vec = pl.vec;
        a.bulk_out = pl.vec && io.xnorm == nullptr;
        a.pf_from = pl.pf_from;
        a.f_k = FastDiv((uint32_t)pl.K);
        a.io = io;
        a.act = act;
        a.err = ds->error_word;
        a.abort_flag = ds->abort_flag;
        a.wait_ns = wait_limit_ns();
        int world = 1;
        if (cv) {
            world = cv->world;
            a.xon = 1;
            a.world = cv->world;
            a.rank = cv->rank;
            a.xpar = (int)(cv->tag & 1u);
            a.xtag = cv->tag;
            a.xcmax = cv->cmax;
            for (int q = 0; q < cv->world; ++q) a.xrec[q] = cv->rec[q];
        } else {
            a.world = 1;
        }
        a.count = (double)batch * (double)spatial * world;
        a.denom = (float)(batch * spatial * world);
        a.cdiv = const_div(a.denom);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)(pl.nc * pl.Q));
        cfg.blockDim = dim3(kCThreads);
        cfg.dynamicSmemBytes = (size_t)dyn_max;
        cfg.stream = stream;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = (unsigned)pl.Q;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        DNB_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
        *launched = true;
        return after_launch(stream, what);
    });
}

template dnb_status run_cluster<false, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                              const char *, const CommView *);
template dnb_status run_cluster<true, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                             const char *, const CommView *);
template dnb_status run_cluster<true, true>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                            const char *, const CommView *);

}  // namespace dnb
