// Fused batchnorm + activation, training forward and backward, staged in shared memory.
//
// The per-channel statistics must be complete before any output element can be written, so
// every element is needed twice: once for the statistics, once for the output. This kernel
// keeps the second use on chip. One persistent CTA per SM holds a ring of "unit" slots in
// shared memory (a unit is U consecutive floats of one (image, channel) plane; with several
// input tensors, a slot holds the unit of each). Channels are taken in groups; every CTA owns
// the same balanced share of each group's units. Per CTA:
//
//   producer warp   streams the share's units of group after group into the ring with TMA
//                   bulk copies (cp.async.bulk, global -> shared, completion on a per-slot
//                   mbarrier; no multicast), as fast as slots come free;
//   stats warps     reduce each unit once it lands (forward: shifted (count, mean, M2) per
//                   lane; backward: sum g and sum g*(x - mean), g = delta * act'(y)) and leave
//                   one partial per warp and channel segment per group;
//   publisher warp  combines a group's per-warp partials and stores the CTA's tagged records
//                   (with a communicator: into every rank's exchange buffer over NVLink);
//   merger warp     polls the records of its share's channels, merges them in fp64 in a fixed
//                   order, and publishes the group's apply parameters in shared memory;
//   apply warps     write the outputs of each unit straight from its slot (forward: y and
//                   optionally x_norm; backward: dx), then free the slot for the producer.
//
// So every input byte crosses HBM exactly once, every output byte once, and the ring holds
// the next groups' units while a group's records are exchanged: HBM keeps streaming through
// the exchange. The groups are sized so that three groups' shares fit the ring. Waits are
// bounded (%globaltimer); a CTA that gives up sets the device error word and the abort flag,
// stops its warps, waits for its own bulk copies to land, and exits.
//
// Reference sequence this replaces: batchnorm.zig:129-174 with the activation of
// convolutional.zig:269/280 (about 56 bytes of HBM traffic per element in each direction,
// against 8 forward and 12 backward here).
#include <atomic>

#include "dnb_bn.cuh"

namespace dnb {
namespace {

constexpr int kTStats = 6;                          // statistics warps
constexpr int kTApply = 8;                          // output warps
constexpr int kTWarps = 1 + kTStats + kTApply + 2;  // + producer, publisher, merger
constexpr int kTThreads = 32 * kTWarps;
constexpr int kTWarpStats0 = 1;
constexpr int kTWarpApply0 = kTWarpStats0 + kTStats;
constexpr int kTWarpPublish = kTWarpApply0 + kTApply;
constexpr int kTWarpMerge = kTWarpPublish + 1;
constexpr int kTGroupRing = 8;  // per-group state buffers: the producer stays fewer groups ahead
constexpr int kTMaxSlots = 256;
constexpr int kTMaxUnitFloats = 2048;  // preferred unit size: at most 8 KB per tensor
constexpr int kTStaticSmemReserve = 1024;  // the kernel's static shared variables fit in this

struct TArgs {
    // partition, as the sweep's (share_of / owner_of)
    int64_t C, S;
    int N, K, U, NK, cg, G, Ps, cap_units;
    uint32_t T_full, T_last;
    FastDiv f_nk, f_k, f_ps, f_tfull, f_tlast;
    // ring: R slots of nt tensors x SU floats
    int R, SU, slot_floats, vec;
    int pf_from;     // first group whose share is prefetched into L2 (earlier ones fit the ring)
    int bulk_out;    // outputs leave by bulk copies from the slot (vec units, no x_norm)
    float denom;
    ConstDiv cdiv;  // division by denom, per element
    BnIO io;
    int act;
    unsigned long long *rec;  // this GPU's records [G][Ps][2 segments][4 words]
    size_t rec_words;
    unsigned *sync;  // [0] launch epoch, [1] CTAs finished with it
    unsigned *err, *abort_flag;
    unsigned long long wait_ns;
    int xon, world, rank, xpar, xpmax;
    unsigned xtag;
    unsigned long long *xrec[kMaxRanks];
};

template <bool BWD, int A, bool HASY>
struct Stage {
    static constexpr int NT = BWD ? (HASY ? 3 : 2) : 1;  // input tensors
    static constexpr int kRecWords = BWD ? 2 : 3;

    struct Smem {
        float *ring;      // [R][slot_floats]
        uint64_t *full;   // [R] the slot's unit has landed
        uint64_t *empty;  // [R] the slot's unit has been written out
        float4 *wrec;     // [DG][2 segments][kTStats] per-warp partials
        double2 *lrec;    // [DG][2] merged records
        double *lcnt;     // [DG][2] elements behind the forward's records
        float *ptab;      // [DG][2][8] apply parameters
        // per-channel inputs of every group's (at most two) share channels, [G][2], loaded once
        // in the prologue so that no global load sits on the exchange's path:
        float4 *ctab;     // the closing's inputs: (gamma, beta) or (mean, var, gamma, beta)
        float4 *stab;     // backward: the forward's (mean, inv, gamma, beta) for the statistics
        float2 *otab;     // the accumulated outputs' prior values: (rolling mean, rolling variance)
                          // or (bias_updates, scale_updates)
        uint64_t *tbar;   // the tables are loaded
        // per group-state buffer b = g % kTGroupRing, one phase per group using it
        // (group g waits on phase g / kTGroupRing, parity (g / kTGroupRing) & 1):
        uint64_t *sbar;  // [DG] every statistics warp has left its partials of the group
        uint64_t *pbar;  // [DG] the publisher has stored the group's records
        uint64_t *rbar;  // [DG] the group's apply parameters are in ptab
        uint64_t *abar;  // [DG] every output warp is done with the group
        int *stop;       // set when any wait gave up
    };
    static size_t ctrl_bytes(int R, int G) {
        return (size_t)R * 16 +
               (size_t)kTGroupRing * (2 * kTStats * sizeof(float4) + 2 * sizeof(double2) + 2 * sizeof(double) +
                                      16 * sizeof(float) + 4 * sizeof(uint64_t)) +
               (size_t)G * 2 * (2 * sizeof(float4) + sizeof(float2)) + 64;
    }
    static size_t smem_bytes(int R, int slot_floats, int G) {
        return (size_t)R * slot_floats * sizeof(float) + ctrl_bytes(R, G);
    }
    __device__ static Smem carve(const TArgs &a, unsigned char *raw) {
        Smem s;
        size_t o = 0;
        s.ring = reinterpret_cast<float *>(raw);
        o += (size_t)a.R * a.slot_floats * sizeof(float);
        s.full = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)a.R * 8;
        s.empty = reinterpret_cast<uint64_t *>(raw + o);
        o += (size_t)a.R * 8;
        s.wrec = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)kTGroupRing * 2 * kTStats * sizeof(float4);
        s.lrec = reinterpret_cast<double2 *>(raw + o);
        o += (size_t)kTGroupRing * 2 * sizeof(double2);
        s.lcnt = reinterpret_cast<double *>(raw + o);
        o += (size_t)kTGroupRing * 2 * sizeof(double);
        s.ptab = reinterpret_cast<float *>(raw + o);
        o += (size_t)kTGroupRing * 16 * sizeof(float);
        s.ctab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)a.G * 2 * sizeof(float4);
        s.stab = reinterpret_cast<float4 *>(raw + o);
        o += (size_t)a.G * 2 * sizeof(float4);
        s.otab = reinterpret_cast<float2 *>(raw + o);
        o += (size_t)a.G * 2 * sizeof(float2);
        s.sbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kTGroupRing * sizeof(uint64_t);
        s.pbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kTGroupRing * sizeof(uint64_t);
        s.rbar = reinterpret_cast<uint64_t *>(raw + o);
        o += kTGroupRing * sizeof(uint64_t);
        s.abar = reinterpret_cast<uint64_t *>(raw + o);
        o += kTGroupRing * sizeof(uint64_t);
        s.tbar = reinterpret_cast<uint64_t *>(raw + o);
        o += sizeof(uint64_t);
        s.stop = reinterpret_cast<int *>(raw + o);
        return s;
    }

    // ---- waits (all bounded) ----
    __device__ static void give_up(const TArgs &a, const Smem &s, unsigned bit) {
        atomicOr(a.err, bit);
        atomicExch(a.abort_flag, 1u);
        *reinterpret_cast<volatile int *>(s.stop) = 1;
    }
    __device__ static bool stopped(const Smem &s) { return *reinterpret_cast<const volatile int *>(s.stop) != 0; }
    // whole warp, warp-uniform result: until the mbarrier phase of `parity` has completed
    __device__ static bool wait_bar(const TArgs &a, const Smem &s, uint64_t *bar, unsigned parity) {
        if (__all_sync(0xffffffffu, mbar_test(bar, parity))) return true;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        for (;;) {
            if (__all_sync(0xffffffffu, mbar_test(bar, parity))) return true;
            int quit = 0;
            if ((threadIdx.x & 31) == 0) {
                if (stopped(s)) {
                    quit = 1;
                } else if (global_ns() > deadline) {
                    give_up(a, s, DEVERR_WAIT_BARRIER);
                    quit = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, quit, 0)) return false;
            __nanosleep(64);
        }
    }
    // whole warp: wait for group g's phase of the group barrier array `bars`
    __device__ static bool wait_group(const TArgs &a, const Smem &s, uint64_t *bars, int g) {
        return wait_bar(a, s, &bars[g % kTGroupRing], (unsigned)(g / kTGroupRing) & 1u);
    }
    // whole warp: lane 0 arrives on group g's barrier of `bars` after the warp's
    // shared-memory writes (the arrive releases them to the waiters)
    __device__ static void arrive_group(uint64_t *bars, int g) {
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&bars[g % kTGroupRing]);
        __syncwarp();
    }

    // element offset of unit t of group g (the plan keeps every offset below 2^32)
    __device__ static uint32_t unit_offset(const TArgs &a, int g, uint32_t t) {
        uint32_t cl, rem, n, k;
        a.f_nk.divmod(t, cl, rem);
        a.f_k.divmod(rem, n, k);
        const uint32_t c = (uint32_t)g * (uint32_t)a.cg + cl;
        return ((n * (uint32_t)a.C + c) * (uint32_t)a.S) + k * (uint32_t)a.U;
    }

    // ---- prologue (every warp but the producer) ----
    // The per-channel inputs of every group's share channels into the tables, all loads in
    // flight at once; each warp's lane 0 then arrives on tbar.
    __device__ static void load_tables(const TArgs &a, const Smem &s, int rid) {
        const int t = (int)threadIdx.x - 32, nt = kTThreads - 32;
        for (int i = t; i < 2 * a.G; i += nt) {
            const int g = i >> 1, j = i & 1;
            const Share sh = share_of(a, g, rid, a.f_ps);
            if (j >= sh.nseg) continue;
            const int cl = sh.cfirst + j;
            const int64_t c = (int64_t)sh.c0 + cl;
            // the accumulated outputs are read only by the CTA that writes them
            const bool owner = owner_of(a, g, (uint32_t)cl * a.NK, a.Ps) == rid;
            if (BWD) {
                const float m = a.io.mean_in[c], v = a.io.var_in[c], gm = a.io.scales[c], bt = a.io.biases[c];
                s.ctab[i] = make_float4(m, v, gm, bt);
                // the forward's normalisation (batchnorm.zig:142), to recompute y from x
                s.stab[i] = make_float4(m, 1.0f / (sqrtf(v) + 0.000001f), gm, bt);
                if (owner) s.otab[i] = make_float2(a.io.bias_upd[c], a.io.scale_upd[c]);
            } else {
                s.ctab[i] = make_float4(a.io.scales[c], a.io.biases[c], 0.0f, 0.0f);
                if (owner) s.otab[i] = make_float2(a.io.rmean[c], a.io.rvar[c]);
            }
        }
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(s.tbar);
        __syncwarp();
    }

    // ---- producer warp ----
    // Units are numbered in the CTA's order of groups and units; unit i lives in slot i % R
    // and is that slot's (i / R)-th occupant. The warp issues up to min(32, R) units at once,
    // one per lane: a unit waits for the slot of unit i - R, which belongs to a group at least
    // two groups back (a group's share is at most R / 2 units), so no unit of a batch waits
    // for another unit of the same or a later batch.
    __device__ static void producer(const TArgs &a, const Smem &s, int rid) {
        const int lane = threadIdx.x & 31;
        const uint64_t pol = l2_evict_first();
        const uint32_t width = a.R < 32 ? (uint32_t)a.R : 32u;
        uint32_t i0 = 0;      // the CTA's unit number of the current group's first unit
        uint32_t issued = 0;  // units whose copies have been issued (in unit order)
        bool ok = true;
        for (int g = 0; g < a.G && ok; ++g) {
            // group g reuses the state buffer of group g - kTGroupRing: wait until every output
            // warp is done with that group
            if (g >= kTGroupRing && !wait_group(a, s, s.abar, g - kTGroupRing)) {
                ok = false;
                break;
            }
            const Share sh = share_of(a, g, rid, a.f_ps);
            const uint32_t n_units = sh.t1 - sh.t0;
            for (uint32_t base = 0; base < n_units && ok; base += width) {
                const uint32_t u = base + (uint32_t)lane;
                const bool has = (uint32_t)lane < width && u < n_units;
                const uint32_t i = i0 + u, slot = i % (uint32_t)a.R, use = i / (uint32_t)a.R;
                // every lane's slot free (its previous occupant written out)
                bool free_ = !has || use == 0 || mbar_test(&s.empty[slot], (use - 1) & 1u);
                if (!__all_sync(0xffffffffu, free_)) {
                    const unsigned long long deadline = global_ns() + a.wait_ns;
                    for (;;) {
                        free_ = free_ || mbar_test(&s.empty[slot], (use - 1) & 1u);
                        if (__all_sync(0xffffffffu, free_)) break;
                        int quit = 0;
                        if (lane == 0) {
                            if (stopped(s)) {
                                quit = 1;
                            } else if (global_ns() > deadline) {
                                give_up(a, s, DEVERR_WAIT_BARRIER);
                                quit = 1;
                            }
                        }
                        if (__shfl_sync(0xffffffffu, quit, 0)) {
                            ok = false;
                            break;
                        }
                        __nanosleep(64);
                    }
                    if (!ok) break;  // no unit of this batch was issued
                }
                if (has) {
                    const uint32_t off = unit_offset(a, g, sh.t0 + u);
                    // vec: the unit is 16-byte aligned; otherwise copy the aligned span around it
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
            // Bring the share of group g + 2 into L2 now: its loads are issued only once
            // slots come free, and then come from L2 while HBM streams the groups after it.
            // Groups that fit the ring at the start are loaded at once and need no prefetch.
            const int q = g + 2;
            if (ok && q < a.G && q >= a.pf_from) {
                const Share sq = share_of(a, q, rid, a.f_ps);
                for (uint32_t u = lane; u < sq.t1 - sq.t0; u += 32) {
                    const uint32_t off = unit_offset(a, q, sq.t0 + u);
                    const uint32_t start = a.vec ? off : (off & ~3u);
                    const uint32_t len = a.vec ? (uint32_t)a.U : ((off - start + (uint32_t)a.U + 3u) & ~3u);
                    prefetch_l2(a.io.t0 + start, len * 4);
                    if (NT > 1) prefetch_l2(a.io.t1 + start, len * 4);
                    if (NT > 2) prefetch_l2(a.io.t2 + start, len * 4);
                }
                __syncwarp();
            }
        }
        drain(a, s, issued);
    }

    // Before the CTA may exit, every copy issued into its shared memory must have landed: the
    // current occupants of the slots, i.e. the last R units issued (older ones have been
    // consumed). On the normal path they have landed already or are about to.
    __device__ static void drain(const TArgs &a, const Smem &s, uint32_t issued) {
        const uint32_t first = issued > (uint32_t)a.R ? issued - (uint32_t)a.R : 0u;
        const unsigned long long deadline = global_ns() + a.wait_ns;
        for (uint32_t k = first + (threadIdx.x & 31); k < issued; k += 32) {
            const uint32_t slot = k % (uint32_t)a.R;
            while (!mbar_test(&s.full[slot], (k / (uint32_t)a.R) & 1u) && global_ns() < deadline) {
                __nanosleep(64);
            }
        }
        __syncwarp();
    }

    // ---- statistics warps ----
    __device__ static void stats(const TArgs &a, const Smem &s, int rid, int ws) {
        const int lane = threadIdx.x & 31;
        if (BWD && !wait_bar(a, s, s.tbar, 0)) return;  // the forward's parameters (stab)
        uint32_t i0 = 0;  // the CTA's unit number of the group's first unit
        for (int g = 0; g < a.G; ++g) {
            // a warp without units in the groups ahead would otherwise reach group g while the
            // publisher still reads group g - kTGroupRing's partials from the same buffer
            if (g >= kTGroupRing && !wait_group(a, s, s.pbar, g - kTGroupRing)) return;
            // every statistics warp is done with group g - 1, so every unit of the earlier
            // groups has landed: the previous occupant of each slot this warp waits on below.
            // Without it a warp running a group ahead could test a slot's `full` barrier while
            // the phase of the slot's previous unit is still open, and a parity wait one phase
            // early succeeds at once (stale data in the sums).
            if (g >= 1 && !wait_group(a, s, s.sbar, g - 1)) return;
            const Share sh = share_of(a, g, rid, a.f_ps);
            const int b = g % kTGroupRing;
            const uint32_t n_units = sh.t1 - sh.t0;
            float4 rec[2] = {make_float4(0.0f, 0.0f, 0.0f, 0.0f), make_float4(0.0f, 0.0f, 0.0f, 0.0f)};
            int seg = 0;
            if constexpr (!BWD) {
                Moments mo;
                float4 first = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                for (uint32_t u = ws; u < n_units; u += kTStats) {
                    const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                    if (!wait_bar(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) return;
                    const int useg = sh.t0 + u >= sh.bnd ? 1 : 0;
                    if (useg != seg) {  // warp-uniform, once at most
                        first = mo.warp_summary();
                        mo = Moments();
                        seg = useg;
                    }
                    const float *src = s.ring + (size_t)slot * a.slot_floats;
                    if (a.vec) {
                        const float4 *v4 = reinterpret_cast<const float4 *>(src);
                        const int n4 = a.U >> 2;
#pragma unroll 4
                        for (int k = lane; k < n4; k += 32) mo.add4(v4[k]);
                    } else {
                        const uint32_t o = unit_offset(a, g, sh.t0 + u) & 3u;
                        for (int k = lane; k < a.U; k += 32) mo.add1(src[o + k]);
                    }
                }
                const float4 last = mo.warp_summary();
                rec[0] = seg ? first : last;
                rec[1] = seg ? last : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            } else {
                float s1 = 0.0f, s2 = 0.0f, f1 = 0.0f, f2 = 0.0f;
                for (uint32_t u = ws; u < n_units; u += kTStats) {
                    const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                    if (!wait_bar(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) return;
                    const int useg = sh.t0 + u >= sh.bnd ? 1 : 0;
                    if (useg != seg) {
                        f1 = s1;
                        f2 = s2;
                        s1 = s2 = 0.0f;
                        seg = useg;
                    }
                    const float4 fp = s.stab[2 * g + seg];
                    BwdParam p;
                    p.m = fp.x;
                    p.inv = fp.y;
                    p.g = fp.z;
                    p.b = fp.w;
                    const float *src = s.ring + (size_t)slot * a.slot_floats;
                    if (a.vec) {
                        const float4 *d4 = reinterpret_cast<const float4 *>(src);
                        const float4 *x4 = reinterpret_cast<const float4 *>(src + a.SU);
                        const float4 *y4 = reinterpret_cast<const float4 *>(src + 2 * a.SU);
                        const int n4 = a.U >> 2;
#pragma unroll 2
                        for (int k = lane; k < n4; k += 32) {
                            const float4 d = d4[k], xv = x4[k];
                            const float4 yy = HASY ? y4[k] : xv;
                            const float g0 = bn_grad1<A, HASY>(d.x, xv.x, yy.x, p, a.act);
                            const float g1 = bn_grad1<A, HASY>(d.y, xv.y, yy.y, p, a.act);
                            const float g2 = bn_grad1<A, HASY>(d.z, xv.z, yy.z, p, a.act);
                            const float g3 = bn_grad1<A, HASY>(d.w, xv.w, yy.w, p, a.act);
                            s1 += (g0 + g1) + (g2 + g3);
                            s2 += (g0 * (xv.x - p.m) + g1 * (xv.y - p.m)) + (g2 * (xv.z - p.m) + g3 * (xv.w - p.m));
                        }
                    } else {
                        const uint32_t o = unit_offset(a, g, sh.t0 + u) & 3u;
                        for (int k = lane; k < a.U; k += 32) {
                            const float xv = src[a.SU + o + k];
                            const float gv = bn_grad1<A, HASY>(src[o + k], xv, HASY ? src[2 * a.SU + o + k] : 0.0f, p,
                                                               a.act);
                            s1 += gv;
                            s2 += gv * (xv - p.m);
                        }
                    }
                }
                const float t1 = warp_sum(s1), t2 = warp_sum(s2);
                const float u1 = warp_sum(f1), u2 = warp_sum(f2);
                rec[0] = seg ? make_float4(u1, u2, 0.0f, 0.0f) : make_float4(t1, t2, 0.0f, 0.0f);
                rec[1] = seg ? make_float4(t1, t2, 0.0f, 0.0f) : make_float4(0.0f, 0.0f, 0.0f, 0.0f);
            }
            if (lane == 0) {
                s.wrec[(2 * b + 0) * kTStats + ws] = rec[0];
                s.wrec[(2 * b + 1) * kTStats + ws] = rec[1];
            }
            arrive_group(s.sbar, g);
            i0 += n_units;
        }
    }

    // first word of the record (group g, segment j) of CTA p of rank r in an exchange buffer
    __device__ static size_t xslot(const TArgs &a, int g, int r, int p, int j) {
        return (((((size_t)a.xpar * kMaxSweepGroups + g) * a.world + r) * a.xpmax + p) * 2 + j) * 4;
    }

    // ---- publisher warp ----
    __device__ static void publisher(const TArgs &a, const Smem &s, int rid, unsigned tag) {
        const int lane = threadIdx.x & 31;
        for (int g = 0; g < a.G; ++g) {
            if (!wait_group(a, s, s.sbar, g)) return;
            const Share sh = share_of(a, g, rid, a.f_ps);
            const int b = g % kTGroupRing;
            for (int j = 0; j < sh.nseg; ++j) {
                float4 q = lane < kTStats ? s.wrec[(2 * b + j) * kTStats + lane] : make_float4(0, 0, 0, 0);
                if constexpr (!BWD) {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        const float cb = __shfl_xor_sync(0xffffffffu, q.x, o);
                        const float mb = __shfl_xor_sync(0xffffffffu, q.y, o);
                        const float qb = __shfl_xor_sync(0xffffffffu, q.z, o);
                        chan_merge(q.x, q.y, q.z, cb, mb, qb);
                    }
                } else {
#pragma unroll
                    for (int o = 16; o > 0; o >>= 1) {
                        q.x += __shfl_xor_sync(0xffffffffu, q.x, o);
                        q.y += __shfl_xor_sync(0xffffffffu, q.y, o);
                    }
                }
                if (a.xon) {
                    // lane 0's record to every rank (the butterfly's lanes differ in the last bits)
                    q.x = __shfl_sync(0xffffffffu, q.x, 0);
                    q.y = __shfl_sync(0xffffffffu, q.y, 0);
                    q.z = __shfl_sync(0xffffffffu, q.z, 0);
                    q.w = __shfl_sync(0xffffffffu, q.w, 0);
                    if (lane < a.world) st_record<kRecWords>(a.xrec[lane] + xslot(a, g, a.rank, rid, j), q, tag, true);
                } else if (lane == 0) {
                    st_record<kRecWords>(a.rec + (((size_t)g * a.Ps + rid) * 2 + j) * 4, q, tag, false);
                }
            }
            arrive_group(s.pbar, g);
        }
    }

    // ---- merger warp ----
    // Merges the records of the (at most two) channels of CTA rid's share of group g into
    // lrec[b]: this GPU's CTAs' records, or with a communicator every rank's, in the same order
    // on every rank. Records of CTAs that hold no unit of the channel are skipped.
    __device__ static bool merge(const TArgs &a, const Smem &s, int g, int rid, unsigned tag) {
        const Share sh = share_of(a, g, rid, a.f_ps);
        const int lane = threadIdx.x & 31;
        const int b = g % kTGroupRing;
        for (int j = 0; j < sh.nseg; ++j) {
            const int cl = sh.cfirst + j;
            const uint32_t ua = (uint32_t)cl * a.NK, ub = ua + a.NK;
            const int plo = owner_of(a, g, ua, a.Ps), phi = owner_of(a, g, ub - 1, a.Ps);
            const int per_rank = phi - plo + 1;
            const int nrec = a.xon ? per_rank * a.world : per_rank;
            // 1: loaded and complete; 0: no record to merge; -1: not yet written
            auto load = [&](int idx, float4 &dst) -> int {
                int q = 0, k = idx;
                if (a.xon) {
                    q = idx / per_rank;
                    k = idx - q * per_rank;
                }
                const int p = plo + k;
                const Share o = share_of(a, g, p, a.f_ps);
                const uint32_t lo = ua > o.t0 ? ua : o.t0, hi = ub < o.t1 ? ub : o.t1;
                if (hi <= lo) return 0;
                const int oj = cl - o.cfirst;
                const bool done =
                    a.xon ? ld_record<kRecWords>(a.xrec[a.rank] + xslot(a, g, q, p, oj), tag, true, dst)
                          : ld_record<kRecWords>(a.rec + (((size_t)g * a.Ps + p) * 2 + oj) * 4, tag, false, dst);
                return done ? 1 : -1;
            };
            constexpr int RL = 4;  // records held per lane: one round trip up to 128 records
            float4 r[RL];
            bool have[RL];
            {
                const unsigned long long deadline = global_ns() + a.wait_ns;
                unsigned polls = 0;
                for (;;) {
                    bool complete = true;
#pragma unroll
                    for (int k = 0; k < RL; ++k) {
                        const int idx = lane + 32 * k;
                        const int st = idx < nrec ? load(idx, r[k]) : 0;
                        have[k] = st == 1;
                        complete = complete && st >= 0;
                    }
                    for (int idx = lane + 32 * RL; idx < nrec; idx += 32) {
                        float4 t;
                        complete = complete && load(idx, t) >= 0;
                    }
                    if (__all_sync(0xffffffffu, complete)) break;
                    int quit = 0;
                    if (lane == 0) {
                        if ((++polls & 7u) == 0 && (ld_volatile(a.abort_flag) || stopped(s))) quit = 1;
                        if (global_ns() > deadline) {
                            give_up(a, s, a.xon ? DEVERR_WAIT_PEER : DEVERR_WAIT_BARRIER);
                            quit = 1;
                        }
                    }
                    if (__shfl_sync(0xffffffffu, quit, 0)) return false;
                    __nanosleep(64);
                }
            }
            double2 mine;
            if constexpr (!BWD) {
                double sn = 0.0, smn = 0.0;
#pragma unroll
                for (int k = 0; k < RL; ++k)
                    if (have[k]) {
                        sn += (double)r[k].x;
                        smn += (double)r[k].x * (double)r[k].y;
                    }
                for (int idx = lane + 32 * RL; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    sn += (double)t.x;
                    smn += (double)t.x * (double)t.y;
                }
                sn = warp_sum(sn);
                const double mu = warp_sum(smn) / sn;
                double m2 = 0.0;
#pragma unroll
                for (int k = 0; k < RL; ++k)
                    if (have[k]) {
                        const double d = (double)r[k].y - mu;
                        m2 += (double)r[k].z + (double)r[k].x * d * d;
                    }
                for (int idx = lane + 32 * RL; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    const double d = (double)t.y - mu;
                    m2 += (double)t.z + (double)t.x * d * d;
                }
                m2 = warp_sum(m2);
                mine = make_double2(mu, m2);
                if (lane == 0) s.lcnt[2 * b + j] = sn;
            } else {
                double s1 = 0.0, s2 = 0.0;
#pragma unroll
                for (int k = 0; k < RL; ++k)
                    if (have[k]) {
                        s1 += (double)r[k].x;
                        s2 += (double)r[k].y;
                    }
                for (int idx = lane + 32 * RL; idx < nrec; idx += 32) {
                    float4 t;
                    if (load(idx, t) != 1) continue;
                    s1 += (double)t.x;
                    s2 += (double)t.y;
                }
                mine = make_double2(warp_sum(s1), warp_sum(s2));
            }
            if (lane == 0) s.lrec[2 * b + j] = mine;
        }
        __syncwarp();
        return true;
    }

    __device__ static void merger(const TArgs &a, const Smem &s, int rid, unsigned tag) {
        const int lane = threadIdx.x & 31;
        if (!wait_bar(a, s, s.tbar, 0)) return;
        for (int g = 0; g < a.G; ++g) {
            const Share sh = share_of(a, g, rid, a.f_ps);
            const int b = g % kTGroupRing;
            if (!merge(a, s, g, rid, tag)) {
                // another CTA (or rank) gave up, or this wait did: stop this CTA's warps too
                if (lane == 0) *reinterpret_cast<volatile int *>(s.stop) = 1;
                return;
            }
            if (lane == 0)
                for (int j = 0; j < sh.nseg; ++j) {
                    const double2 tot = s.lrec[2 * b + j];
                    const float4 ci = s.ctab[2 * g + j];
                    float *out = s.ptab + (2 * b + j) * 8;
                    if constexpr (!BWD) {
                        const FwdClose f = fwd_close(tot.x, tot.y, s.lcnt[2 * b + j]);
                        *reinterpret_cast<float4 *>(out) = make_float4(f.m, f.inv, ci.x, ci.y);
                    } else {
                        *reinterpret_cast<BwdParam *>(out) = bwd_params(tot.x, tot.y, ci.x, ci.y, ci.z, ci.w, a.denom);
                    }
                }
            arrive_group(s.rbar, g);
            // the per-channel outputs, by the CTA that owns the channel's first unit
            if (lane == 0)
                for (int j = 0; j < sh.nseg; ++j) {
                    const int cl = sh.cfirst + j;
                    const int64_t c = (int64_t)sh.c0 + cl;
                    if (owner_of(a, g, (uint32_t)cl * a.NK, a.Ps) != rid) continue;
                    const double2 tot = s.lrec[2 * b + j];
                    const float2 prior = s.otab[2 * g + j];  // read in the prologue; this CTA alone writes c
                    if constexpr (!BWD) {
                        const FwdClose f = fwd_close(tot.x, tot.y, s.lcnt[2 * b + j]);
                        a.io.mean[c] = f.m;
                        a.io.var[c] = f.var;
                        a.io.rmean[c] = rolling(prior.x, f.m);
                        a.io.rvar[c] = rolling(prior.y, f.var);
                    } else {
                        const float4 ci = s.ctab[2 * g + j];
                        float md;
                        const BwdParam p = bwd_params(tot.x, tot.y, ci.x, ci.y, ci.z, ci.w, a.denom, &md);
                        // bwd_write's accumulation, on the prior values
                        a.io.bias_upd[c] = prior.x + (float)tot.x;
                        a.io.scale_upd[c] = prior.y + (float)(tot.y * (double)p.inv);
                        a.io.mean_delta[c] = md;
                        a.io.var_delta[c] = p.vd;
                    }
                }
            __syncwarp();
        }
    }

    // ---- output warps ----
    // With a.bulk_out the outputs are written over the unit's first tensor in its slot and
    // leave by one bulk copy per unit (lane 0's bulk groups, one per unit); the slot returns
    // to the producer once that copy has read it, which lane 0 checks one unit later (or at
    // the group's end, so that no slot stays held while the warp waits for the next group).
    // Otherwise the lanes store the outputs themselves and the slot returns at once.
    __device__ static void apply(const TArgs &a, const Smem &s, int rid, int wa) {
        const int lane = threadIdx.x & 31;
        uint32_t i0 = 0;
        int held = -1;  // lane 0: the slot whose bulk copy may still read it
        for (int g = 0; g < a.G; ++g) {
            const Share sh = share_of(a, g, rid, a.f_ps);
            const int b = g % kTGroupRing;
            const uint32_t n_units = sh.t1 - sh.t0;
            // every output warp waits for the group's parameters, also one without units in it:
            // its arrival on abar below must not count towards an earlier group's phase (the
            // producer reuses the group's state buffer once that phase completes)
            if (!wait_group(a, s, s.rbar, g)) break;
            bool ok = true;
            for (uint32_t u = wa; u < n_units; u += kTApply) {
                const uint32_t i = i0 + u, slot = i % (uint32_t)a.R;
                // already complete (the statistics waited on it): the acquire of its data
                if (!wait_bar(a, s, &s.full[slot], (i / (uint32_t)a.R) & 1u)) {
                    ok = false;
                    break;
                }
                const int seg = sh.t0 + u >= sh.bnd ? 1 : 0;
                const float *pt = s.ptab + (2 * b + seg) * 8;
                const uint32_t off = unit_offset(a, g, sh.t0 + u);
                float *src = s.ring + (size_t)slot * a.slot_floats;
                if constexpr (!BWD) {
                    const float4 p = *reinterpret_cast<const float4 *>(pt);
                    if (a.bulk_out) {
                        float4 *v4 = reinterpret_cast<float4 *>(src);
                        const int n4 = a.U >> 2;
#pragma unroll 4
                        for (int k = lane; k < n4; k += 32) {
                            const float4 v = v4[k];
                            v4[k] = make_float4(bn_fwd1<A>(v.x, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.y, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.z, p.x, p.y, p.z, p.w, a.act),
                                                bn_fwd1<A>(v.w, p.x, p.y, p.z, p.w, a.act));
                        }
                    } else if (a.vec) {
                        const float4 *v4 = reinterpret_cast<const float4 *>(src);
                        const int n4 = a.U >> 2;
                        float *dst = a.io.out + off;
#pragma unroll 4
                        for (int k = lane; k < n4; k += 32) {
                            const float4 v = v4[k];
                            if (a.io.xnorm)
                                st4(a.io.xnorm + off + 4 * k, make_float4((v.x - p.x) * p.y, (v.y - p.x) * p.y,
                                                                          (v.z - p.x) * p.y, (v.w - p.x) * p.y));
                            st4(dst + 4 * k, make_float4(bn_fwd1<A>(v.x, p.x, p.y, p.z, p.w, a.act),
                                                         bn_fwd1<A>(v.y, p.x, p.y, p.z, p.w, a.act),
                                                         bn_fwd1<A>(v.z, p.x, p.y, p.z, p.w, a.act),
                                                         bn_fwd1<A>(v.w, p.x, p.y, p.z, p.w, a.act)));
                        }
                    } else {
                        const uint32_t o = off & 3u;
                        for (int k = lane; k < a.U; k += 32) {
                            const float v = src[o + k];
                            if (a.io.xnorm) a.io.xnorm[off + k] = (v - p.x) * p.y;
                            a.io.out[off + k] = bn_fwd1<A>(v, p.x, p.y, p.z, p.w, a.act);
                        }
                    }
                } else {
                    const BwdParam p = *reinterpret_cast<const BwdParam *>(pt);
                    if (a.vec) {
                        float4 *d4 = reinterpret_cast<float4 *>(src);
                        const float4 *x4 = reinterpret_cast<const float4 *>(src + a.SU);
                        const float4 *y4 = reinterpret_cast<const float4 *>(src + 2 * a.SU);
                        const int n4 = a.U >> 2;
                        float *dst = a.io.out + off;
#pragma unroll 2
                        for (int k = lane; k < n4; k += 32) {
                            const float4 d = d4[k], xv = x4[k];
                            const float4 yy = HASY ? y4[k] : xv;
                            const float4 r = bn_dx4_p(bn_grad4<A, HASY>(d, xv, yy, p, a.act), xv, p, a);
                            if (a.bulk_out)
                                d4[k] = r;  // over delta, element by element
                            else
                                st4(dst + 4 * k, r);
                        }
                    } else {
                        const uint32_t o = off & 3u;
                        for (int k = lane; k < a.U; k += 32) {
                            const float xv = src[a.SU + o + k];
                            const float gv =
                                bn_grad1<A, HASY>(src[o + k], xv, HASY ? src[2 * a.SU + o + k] : 0.0f, p, a.act);
                            a.io.out[off + k] = bn_dx_p(gv, xv, p, a);
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
                    // the unit's slot is read: hand it back to the producer
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
            arrive_group(s.abar, g);
            i0 += n_units;
        }
        // every bulk copy of this warp complete (read from the slots and written out) before
        // the CTA may end
        if (lane == 0) bulk_wait_all();
        __syncwarp();
    }
};

template <bool BWD, int A, bool HASY>
__global__ void __launch_bounds__(kTThreads, 1) k_bn_stage(TArgs a) {
    using K = Stage<BWD, A, HASY>;
    extern __shared__ __align__(128) unsigned char smem_raw[];
    const typename K::Smem s = K::carve(a, smem_raw);
    __shared__ unsigned s_epoch;
    __shared__ int s_exited;
    const int rid = (int)blockIdx.x;
    if (threadIdx.x == 0) {
        s_epoch = ld_volatile(&a.sync[0]);
        *s.stop = 0;
        s_exited = 0;
    }
    if (threadIdx.x == 0) mbar_init(s.tbar, kTWarps - 1);
    if (threadIdx.x < kTGroupRing) {
        mbar_init(&s.sbar[threadIdx.x], kTStats);
        mbar_init(&s.pbar[threadIdx.x], 1);
        mbar_init(&s.rbar[threadIdx.x], 1);
        mbar_init(&s.abar[threadIdx.x], kTApply);
    }
    for (int i = threadIdx.x; i < a.R; i += kTThreads) {
        mbar_init(&s.full[i], 1);
        mbar_init(&s.empty[i], 1);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncthreads();
    const unsigned epoch = s_epoch;
    const unsigned tag = a.xon ? a.xtag : epoch + 1u;  // never 0, the tag of a cleared record
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    // the epoch advances once per launch, after every CTA has read it (the last publisher to
    // finish does it); in the launch whose successor's tag would wrap to 0, the last warp of
    // the last CTA clears the record area instead (once per 2^32 - 1 launches)
    const bool wraps = epoch + 2u == 0u;
    if (warp != 0) K::load_tables(a, s, rid);
    if (warp == 0) {
        K::producer(a, s, rid);
    } else if (warp < kTWarpApply0) {
        K::stats(a, s, rid, warp - kTWarpStats0);
    } else if (warp < kTWarpPublish) {
        K::apply(a, s, rid, warp - kTWarpApply0);
    } else if (warp == kTWarpPublish) {
        K::publisher(a, s, rid, tag);
        __syncwarp();
        if (!wraps && lane == 0 && atomicAdd(&a.sync[1], 1u) == (unsigned)a.Ps - 1u) {
            a.sync[1] = 0u;
            a.sync[0] = epoch + 1u;
        }
    } else if (warp == kTWarpMerge) {
        K::merger(a, s, rid, tag);
    }
    if (!wraps) return;
    __syncwarp();
    int last = 0;
    if (lane == 0 && atomicAdd(&s_exited, 1) == kTWarps - 1) last = atomicAdd(&a.sync[1], 1u) == (unsigned)a.Ps - 1u;
    if (!__shfl_sync(0xffffffffu, last, 0)) return;
    for (size_t i = lane; i < a.rec_words; i += 32) a.rec[i] = 0ull;
    __syncwarp();
    if (lane == 0) {
        a.sync[1] = 0u;
        a.sync[0] = 0u;
    }
}

struct TPlan {
    bool ok = false;
    int K = 0, U = 0, SU = 0, cg = 0, G = 0, cap = 0, R = 0, vec = 0, pf_from = 0;
    size_t smem = 0;
};

// Units of U = spatial / K floats (K the smallest divisor keeping U a multiple of 4 and at
// most kTMaxUnitFloats; a whole plane when spatial % 4 != 0); R slots fill the shared memory a
// CTA may opt into; the channel groups are as large as keeps three groups' shares (two if
// three do not fit) within the ring, so that a group's exchange overlaps the next groups'
// loads.
template <bool BWD, bool HASY>
TPlan plan_stage(int64_t batch, int64_t filters, int64_t spatial, int P, size_t smem_avail) {
    constexpr int nt = BWD ? (HASY ? 3 : 2) : 1;
    using KS = Stage<BWD, DNB_ACT_LEAKY, HASY>;
    TPlan pl;
    if (batch <= 0 || filters <= 0 || spatial <= 0 || P <= 0) return pl;
    if ((uint64_t)batch * (uint64_t)filters * (uint64_t)spatial >= (1ull << 32) - 8) return pl;  // 32-bit offsets
    pl.vec = spatial % 4 == 0;
    if (pl.vec) {
        int64_t k = 0;
        for (int64_t kk = 1; kk <= spatial / 4; ++kk) {
            if (spatial % kk || (spatial / kk) % 4) continue;
            if (spatial / kk <= kTMaxUnitFloats) {
                k = kk;
                break;
            }
        }
        if (k == 0) k = 1;  // no divisor gives a small unit: whole planes
        pl.K = (int)k;
        pl.U = (int)(spatial / k);
        pl.SU = pl.U;
    } else {
        // the aligned span of a plane may reach up to 3 floats past the tensor's end: only
        // when the element count is a multiple of 4 does that stay inside the tensor
        if ((batch * filters * spatial) % 4 != 0) return pl;
        pl.K = 1;
        pl.U = (int)spatial;
        pl.SU = (int)((spatial + 3 + 3) & ~(int64_t)3);
    }
    const size_t slot_bytes = (size_t)nt * pl.SU * sizeof(float);
    int R = 0;
    for (int r = kTMaxSlots; r >= 2; --r)
        if (KS::smem_bytes(r, nt * pl.SU, kMaxSweepGroups) <= smem_avail) {
            R = r;
            break;
        }
    if (R < 2 || slot_bytes * 2 > smem_avail) return pl;
    const int64_t NK = batch * pl.K;
    // a tensor whose shares all fit the ring at once is one group: one exchange in all
    {
        const int64_t T = filters * NK;
        const int64_t cap = (T + P - 1) / P;
        if (filters <= P && cap <= R && (uint64_t)T * (uint64_t)P < (1ull << 32) - (uint64_t)P) {
            pl.cg = (int)filters;
            pl.G = 1;
            pl.cap = (int)cap;
            pl.R = R;
            pl.smem = KS::smem_bytes(R, nt * pl.SU, 1);
            pl.pf_from = 1;
            pl.ok = true;
            return pl;
        }
    }
    for (int D = 3; D >= 2 && !pl.ok; --D) {
        const int64_t capmax = R / D;
        if (capmax < 1) continue;
        int64_t cg = capmax * P / NK;
        if (cg < 1) continue;
        if (cg > P) cg = P;
        if (cg > filters) cg = filters;
        int64_t G = (filters + cg - 1) / cg;
        cg = (filters + G - 1) / G;
        G = (filters + cg - 1) / cg;
        if (G > kMaxSweepGroups) return pl;
        const int64_t T = cg * NK;
        if ((uint64_t)T * (uint64_t)P >= (1ull << 32) - (uint64_t)P) return pl;
        pl.cg = (int)cg;
        pl.G = (int)G;
        pl.cap = (int)((T + P - 1) / P);
        pl.R = R;
        pl.smem = KS::smem_bytes(R, nt * pl.SU, pl.G);
        pl.pf_from = pl.cap > 0 ? R / pl.cap : pl.G;
        pl.ok = true;
    }
    return pl;
}

}  // namespace

bool stage_disabled() {
    const char *e = getenv("DNB_BN_STAGE");
    return e && e[0] == '0';
}

template <bool BWD, bool HASY>
dnb_status run_stage(int64_t batch, int64_t filters, int64_t spatial, int act, const BnIO &io, cudaStream_t stream,
                     bool *launched, const char *what, const CommView *cv) {
    *launched = false;
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    // every tensor the bulk copies and the vector stores touch starts 16-byte aligned
    const void *ins[3] = {io.t0, io.t1, io.t2};
    for (int k = 0; k < (BWD ? (HASY ? 3 : 2) : 1); ++k)
        if (!aligned16(ins[k])) return DNB_OK;
    if (!aligned16(io.out) || (io.xnorm && !aligned16(io.xnorm))) return DNB_OK;
    const int P = ds->sm_count;
    // dynamic shared memory: what a CTA may opt into, less room for the kernel's own static
    // variables
    const int dyn_max = ds->max_smem_optin - kTStaticSmemReserve;
    const TPlan pl = plan_stage<BWD, HASY>(batch, filters, spatial, P, (size_t)dyn_max);
    if (!pl.ok) return DNB_OK;
    if (cv && (P > cv->pmax || pl.G > kMaxSweepGroups)) return DNB_OK;
    return dispatch_act(act, [&]<int A>() -> dnb_status {
        auto kern = k_bn_stage<BWD, A, HASY>;
        // per device: the opt-in shared memory limit, set once to the most a CTA may take, and
        // whether one CTA of that size fits an SM (cached as 1 + yes)
        static std::atomic<int> ready_by_device[kMaxDevices];
        int r1 = ready_by_device[ds->device].load(std::memory_order_relaxed);
        if (r1 == 0) {
            DNB_CUDA(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, dyn_max));
            int occ = 0;
            DNB_CUDA(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, kern, kTThreads, dyn_max));
            r1 = occ >= 1 ? 2 : 1;
            ready_by_device[ds->device].store(r1, std::memory_order_relaxed);
        }
        if (r1 != 2) return DNB_OK;
        Workspace *ws = nullptr;
        DNB_TRY(workspace(stream, 0, &ws, (size_t)pl.G * P * 2 * 4));
        TArgs a{};
        a.C = filters;
        a.S = spatial;
        a.N = (int)batch;
        a.K = pl.K;
        a.U = pl.U;
        a.NK = (int)(batch * pl.K);
        a.cg = pl.cg;
        a.G = pl.G;
        a.Ps = P;
        a.cap_units = pl.cap;
        a.T_full = (uint32_t)pl.cg * (uint32_t)a.NK;
        a.T_last = (uint32_t)(filters - (int64_t)(pl.G - 1) * pl.cg) * (uint32_t)a.NK;
        a.f_nk = FastDiv((uint32_t)a.NK);
        a.f_k = FastDiv((uint32_t)pl.K);
        a.f_ps = FastDiv((uint32_t)P);
        a.f_tfull = FastDiv(a.T_full);
        a.f_tlast = FastDiv(a.T_last);
        a.R = pl.R;
        a.SU = pl.SU;
        a.slot_floats = (BWD ? (HASY ? 3 : 2) : 1) * pl.SU;
        a.vec = pl.vec;
        a.pf_from = pl.pf_from;
        a.bulk_out = pl.vec && io.xnorm == nullptr;
        a.io = io;
        a.act = act;
        a.rec = ws->recs;
        a.rec_words = ws->rec_words;
        a.sync = ws->sync;
        a.err = ds->error_word;
        a.abort_flag = ds->abort_flag;
        a.wait_ns = wait_limit_ns();
        a.xon = 0;
        a.world = 1;
        int64_t count = batch * spatial;
        if (cv) {
            a.xon = 1;
            a.world = cv->world;
            a.rank = cv->rank;
            a.xpar = (int)(cv->tag & 1u);
            a.xpmax = cv->pmax;
            a.xtag = cv->tag;
            for (int r = 0; r < cv->world; ++r) a.xrec[r] = cv->rec[r];
            count *= cv->world;  // normalize_delta divides by the element count of the whole batch
        }
        a.denom = (float)count;
        a.cdiv = const_div(a.denom);
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3((unsigned)P);
        cfg.blockDim = dim3(kTThreads);
        cfg.dynamicSmemBytes = pl.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        DNB_CUDA(cudaLaunchKernelEx(&cfg, kern, a));
        *launched = true;
        return after_launch(stream, what);
    });
}

template dnb_status run_stage<false, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                            const char *, const CommView *);
template dnb_status run_stage<true, false>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                           const char *, const CommView *);
template dnb_status run_stage<true, true>(int64_t, int64_t, int64_t, int, const BnIO &, cudaStream_t, bool *,
                                          const char *, const CommView *);

}  // namespace dnb
