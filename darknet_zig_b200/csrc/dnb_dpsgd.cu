// Data-parallel weight update in one kernel per rank, over NVLink peer memory.
//
// The reference updates a layer's weights on its one GPU (convolutional.zig:330-334:
// axpy(-decay*batch, w, wu), axpy(lr/batch, wu, w), scal(momentum, wu), with wu the
// gradients accumulated by the backward pass). With N data-parallel ranks the update needs
// the sum of every rank's gradients. The usual form is three steps: a reduce-scatter of the
// gradients, the update of each rank's shard, an all-gather of the weights. Here one kernel
// does all three, element by element: rank r owns 1/N of the weights; for each element of its
// shard it loads the gradient from every rank's buffer (plain peer loads, added in rank order
// so every element has one defined value), adds it into its momentum shard, applies the fused
// SGD, and stores the new weight into every rank's weight vector (plain peer stores). The
// transfers overlap the arithmetic, and the gradient and weight vectors cross NVLink once
// each way.
//
// The weight and gradient vectors live in one library allocation per rank, shared with the
// other ranks through CUDA IPC (the 64-byte handle is swapped by the host once). A small flag
// area in the same allocation carries the call number: a kernel announces its start to every
// rank (its gradients are complete and its weights no longer read by this step) and waits for
// every rank's announcement before touching peer memory; its last CTA announces the end to
// every rank and waits for every rank's end (their stores into this rank's weights are done
// and they no longer read its gradients) before the kernel ends. Every wait is bounded and
// reports through the device error word; after a timeout the group must be recreated.
#include <string.h>

#include "dnb_common.cuh"

namespace dnb {
namespace {

constexpr int kDpThreads = 256;

struct DpGroup {
    int rank = 0, world = 1, device = 0;
    int64_t n = 0, shard = 0, n_pad = 0;
    size_t bytes = 0;
    void *local = nullptr;
    char *peer[kMaxRanks] = {};  // every rank's allocation (peer[rank] = local)
    unsigned *counter = nullptr;  // CTAs of the current call that are done (this rank)
    unsigned calls = 0;
    bool connected = false;
};

// Allocation of one rank: [weights: n_pad floats][gradients: n_pad floats][flags: 2 x kMaxRanks
// 64-bit words: start[q], then end[q], each the call number rank q wrote last].
inline size_t flags_offset(int64_t n_pad) { return (size_t)n_pad * 2 * sizeof(float); }

struct DpArgs {
    int rank, world;
    int64_t lo, shard;  // this rank's shard [lo, lo + shard), shard a multiple of 4
    const float *grads[kMaxRanks];
    float *weights[kMaxRanks];
    unsigned long long *flags[kMaxRanks];
    float *wu;  // this rank's momentum shard
    float a_decay, a_lr, mom;
    unsigned long long tag;
    unsigned *counter;
    unsigned *err, *abort_flag;
    unsigned long long wait_ns;
};

__device__ __forceinline__ void st_flag(unsigned long long *p, unsigned long long v) {
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_flag(const unsigned long long *p) {
    unsigned long long v;
    asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
// one thread: until every rank's flag at `base + q` carries the tag (bounded)
__device__ bool wait_flags(const DpArgs &a, const unsigned long long *base) {
    const unsigned long long deadline = global_ns() + a.wait_ns;
    for (;;) {
        bool all = true;
        for (int q = 0; q < a.world; ++q) all = all && ld_flag(base + q) == a.tag;
        if (all) return true;
        if (ld_volatile(a.abort_flag)) return false;
        if (global_ns() > deadline) {
            atomicOr(a.err, DEVERR_WAIT_PEER);
            atomicExch(a.abort_flag, 1u);
            return false;
        }
        __nanosleep(128);
    }
}

// y = sgd of one element: the fused update of dnb_sgd_momentum after wu += g
__device__ __forceinline__ void dp_update1(float &w, float &u, float g, const DpArgs &a) {
    u = __fmaf_rn(1.0f, g, u);             // axpy(1, g, wu): the gradient into the momentum
    u = __fmaf_rn(a.a_decay, w, u);        // axpy(-decay*batch, w, wu)
    w = __fmaf_rn(a.a_lr, u, w);           // axpy(lr/batch, wu, w)
    u = u * a.mom;                         // scal(momentum, wu)
}

__global__ void __launch_bounds__(kDpThreads) k_dpsgd(DpArgs a) {
    __shared__ int s_ok, s_last;
    // this rank's start, announced to every rank once per call
    if (blockIdx.x == 0 && threadIdx.x < a.world) st_flag(a.flags[threadIdx.x] + a.rank, a.tag);
    if (threadIdx.x == 0) s_ok = wait_flags(a, a.flags[a.rank]);
    __syncthreads();
    if (s_ok) {
        const int64_t n4 = a.shard >> 2;
        for (int64_t k = (int64_t)blockIdx.x * kDpThreads + threadIdx.x; k < n4; k += (int64_t)gridDim.x * kDpThreads) {
            const int64_t i = a.lo + 4 * k;
            float4 g = ld4(a.grads[0] + i);
            for (int q = 1; q < a.world; ++q) {
                const float4 h = ld4(a.grads[q] + i);
                g.x += h.x;
                g.y += h.y;
                g.z += h.z;
                g.w += h.w;
            }
            float4 w = ld4(a.weights[a.rank] + i);
            float4 u = ld4(a.wu + 4 * k);
            dp_update1(w.x, u.x, g.x, a);
            dp_update1(w.y, u.y, g.y, a);
            dp_update1(w.z, u.z, g.z, a);
            dp_update1(w.w, u.w, g.w, a);
            st4(a.wu + 4 * k, u);
            for (int q = 0; q < a.world; ++q) st4(a.weights[q] + i, w);
        }
    }
    // the last CTA of this rank announces the end to every rank once all CTAs' stores are
    // performed, then waits for every rank's end
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(a.counter, 1u) == gridDim.x - 1u;
    __syncthreads();
    if (!s_last) return;
    __threadfence_system();
    if (threadIdx.x == 0) *a.counter = 0u;
    if (threadIdx.x < a.world) st_flag(a.flags[threadIdx.x] + kMaxRanks + a.rank, a.tag);
    __syncthreads();
    if (threadIdx.x == 0) (void)wait_flags(a, a.flags[a.rank] + kMaxRanks);
}

}  // namespace
}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_dpsgd_init(int rank, int world, int64_t n, void *handle_out, float **weights, float **grads,
                          int64_t *shard_lo, int64_t *shard_n, dnb_dpsgd *group) {
    if (!group || !handle_out || !weights || !grads || !shard_lo || !shard_n)
        return fail(DNB_ERR_INVALID, "dpsgd_init: null pointer");
    *group = nullptr;
    if (world < 1 || world > kMaxRanks) return fail(DNB_ERR_INVALID, "dpsgd_init: world %d not in 1..%d", world, kMaxRanks);
    if (rank < 0 || rank >= world) return fail(DNB_ERR_INVALID, "dpsgd_init: rank %d of %d", rank, world);
    if (n < 1) return fail(DNB_ERR_INVALID, "dpsgd_init: n %lld", (long long)n);
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    DpGroup *g = new DpGroup();
    g->rank = rank;
    g->world = world;
    g->device = ds->device;
    g->n = n;
    g->shard = ((n + world - 1) / world + 3) & ~(int64_t)3;  // a multiple of 4: float4 access
    g->n_pad = g->shard * world;
    g->bytes = flags_offset(g->n_pad) + 2 * kMaxRanks * sizeof(unsigned long long);
    cudaError_t e = cudaMalloc(&g->local, g->bytes);
    if (e == cudaSuccess) e = cudaMemset(g->local, 0, g->bytes);
    if (e == cudaSuccess) e = cudaMalloc(&g->counter, sizeof(unsigned));
    if (e == cudaSuccess) e = cudaMemset(g->counter, 0, sizeof(unsigned));
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, g->local);
    if (e != cudaSuccess) {
        if (g->local) cudaFree(g->local);
        if (g->counter) cudaFree(g->counter);
        delete g;
        return cuda_fail(e, "dpsgd_init: shared buffers", __FILE__, __LINE__);
    }
    memcpy(handle_out, &h, sizeof(h));
    g->peer[rank] = static_cast<char *>(g->local);
    *weights = static_cast<float *>(g->local);
    *grads = static_cast<float *>(g->local) + g->n_pad;
    *shard_lo = (int64_t)rank * g->shard;
    *shard_n = g->shard;
    *group = g;
    return DNB_OK;
}

dnb_status dnb_dpsgd_connect(dnb_dpsgd group, const void *handles) {
    DpGroup *g = static_cast<DpGroup *>(group);
    if (!g || !handles) return fail(DNB_ERR_INVALID, "dpsgd_connect: null pointer");
    if (g->connected) return DNB_OK;
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    if (device != g->device) return fail(DNB_ERR_INVALID, "dpsgd_connect: group of device %d on device %d", g->device, device);
    for (int r = 0; r < g->world; ++r) {
        if (r == g->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + 64 * (size_t)r, sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != g->rank && g->peer[q]) {
                    cudaIpcCloseMemHandle(g->peer[q]);
                    g->peer[q] = nullptr;
                }
            return cuda_fail(e, "dpsgd_connect: cudaIpcOpenMemHandle", __FILE__, __LINE__);
        }
        g->peer[r] = static_cast<char *>(p);
    }
    g->connected = true;
    return DNB_OK;
}

dnb_status dnb_dpsgd_step(dnb_dpsgd group, float *momentum, float learning_rate, float momentum_coef, float decay,
                          int64_t batch, dnb_stream stream) {
    DpGroup *g = static_cast<DpGroup *>(group);
    if (!g || !momentum) return fail(DNB_ERR_INVALID, "dpsgd_step: null pointer");
    if (!g->connected) return fail(DNB_ERR_NOT_INIT, "dpsgd_step: group not connected (dnb_dpsgd_connect)");
    if (batch <= 0) return fail(DNB_ERR_INVALID, "dpsgd_step: batch must be positive");
    if (!aligned16(momentum)) return fail(DNB_ERR_INVALID, "dpsgd_step: momentum must be 16-byte aligned");
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    if (device != g->device) return fail(DNB_ERR_INVALID, "dpsgd_step: group of device %d on device %d", g->device, device);
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    ++g->calls;
    if (g->calls == 0) g->calls = 1;  // 0 is the flags' value before any call
    DpArgs a{};
    a.rank = g->rank;
    a.world = g->world;
    a.lo = (int64_t)g->rank * g->shard;
    a.shard = g->shard;
    for (int r = 0; r < g->world; ++r) {
        float *base = reinterpret_cast<float *>(g->peer[r]);
        a.weights[r] = base;
        a.grads[r] = base + g->n_pad;
        a.flags[r] = reinterpret_cast<unsigned long long *>(g->peer[r] + flags_offset(g->n_pad));
    }
    a.wu = momentum;
    const float b = (float)batch;  // convolutional.zig:313
    a.a_decay = -decay * b;
    a.a_lr = learning_rate / b;
    a.mom = momentum_coef;
    a.tag = g->calls;
    a.counter = g->counter;
    a.err = ds->error_word;
    a.abort_flag = ds->abort_flag;
    a.wait_ns = wait_limit_ns();
    const cudaStream_t s = as_stream(stream);
    k_dpsgd<<<(unsigned)(ds->sm_count * 4), kDpThreads, 0, s>>>(a);
    return after_launch(s, "dpsgd_step");
}

dnb_status dnb_dpsgd_destroy(dnb_dpsgd group) {
    DpGroup *g = static_cast<DpGroup *>(group);
    if (!g) return DNB_OK;
    DNB_CUDA(cudaDeviceSynchronize());
    for (int r = 0; r < g->world; ++r)
        if (r != g->rank && g->peer[r]) cudaIpcCloseMemHandle(g->peer[r]);
    if (g->local) cudaFree(g->local);
    if (g->counter) cudaFree(g->counter);
    delete g;
    return DNB_OK;
}

}  // extern "C"
