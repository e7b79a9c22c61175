// Sync-BN communicator: each rank's exchange buffer, shared with the other ranks through
// CUDA IPC so that the fused sweep kernel can store its CTAs' per-channel records straight
// into every peer's memory over NVLink. No collective library is on this path; the host only
// swaps the 64-byte IPC handles once (any transport).
//
// Buffer of one rank: tagged records, 64-bit words
// [2 parities][kMaxSweepGroups][world][pmax][2 segments][4]. A launch with call number t
// (never 0; identical on every rank because every rank makes the same calls) uses parity
// t & 1 and tags every word it stores with t; a rank has a record once all its words carry
// t. A rank can start call t+1 while a slower peer still reads the records of call t, never
// call t+2 (that needs the slower peer's records of call t+1). Tags repeat after 2^32 - 1
// calls of one communicator.
#include <string.h>

#include "dnb_common.cuh"

namespace dnb {

struct Comm {
    int rank = 0, world = 1, device = 0, pmax = 0;
    int64_t cmax = 0;
    size_t rec_bytes = 0, bytes = 0;
    void *local = nullptr;
    void *peer[kMaxRanks] = {};  // opened IPC mappings (peer[rank] = local)
    bool connected = false;
    unsigned calls = 0;
};

dnb_status comm_next(dnb_comm handle, CommView *out) {
    Comm *c = static_cast<Comm *>(handle);
    if (!c) return fail(DNB_ERR_INVALID, "sync-BN: null communicator");
    if (!c->connected) return fail(DNB_ERR_NOT_INIT, "sync-BN: communicator not connected (dnb_comm_connect)");
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    if (device != c->device)
        return fail(DNB_ERR_INVALID, "sync-BN: communicator of device %d used on device %d", c->device, device);
    ++c->calls;
    if (c->calls == 0) c->calls = 1;  // 0 is the tag of a buffer nobody wrote
    out->rank = c->rank;
    out->world = c->world;
    out->tag = c->calls;
    out->cmax = c->cmax;
    out->pmax = c->pmax;
    for (int r = 0; r < c->world; ++r) out->rec[r] = static_cast<unsigned long long *>(c->peer[r]);
    return DNB_OK;
}

}  // namespace dnb

using namespace dnb;

extern "C" {

dnb_status dnb_comm_init(int rank, int world, int64_t max_channels, void *handle_out, dnb_comm *comm) {
    if (!comm || !handle_out) return fail(DNB_ERR_INVALID, "comm_init: null pointer");
    *comm = nullptr;
    if (world < 1 || world > kMaxRanks) return fail(DNB_ERR_INVALID, "comm_init: world %d not in 1..%d", world, kMaxRanks);
    if (rank < 0 || rank >= world) return fail(DNB_ERR_INVALID, "comm_init: rank %d of %d", rank, world);
    if (max_channels < 1 || max_channels > 65535) return fail(DNB_ERR_INVALID, "comm_init: max_channels %lld",
                                                            (long long)max_channels);
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    Comm *c = new Comm();
    c->rank = rank;
    c->world = world;
    c->device = ds->device;
    c->cmax = max_channels;
    c->pmax = ds->sm_count * 4;  // the sweep runs at most 4 CTAs per SM
    c->rec_bytes = sizeof(unsigned long long) * 2 * (size_t)kMaxSweepGroups * world * c->pmax * 2 * 4;
    c->bytes = c->rec_bytes;
    cudaError_t e = cudaMalloc(&c->local, c->bytes);
    if (e == cudaSuccess) e = cudaMemset(c->local, 0, c->bytes);
    cudaIpcMemHandle_t h;
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, c->local);
    if (e != cudaSuccess) {
        if (c->local) cudaFree(c->local);
        delete c;
        return cuda_fail(e, "comm_init: exchange buffer", __FILE__, __LINE__);
    }
    static_assert(sizeof(cudaIpcMemHandle_t) == 64, "IPC handle size");
    memcpy(handle_out, &h, sizeof(h));
    c->peer[rank] = c->local;
    *comm = c;
    return DNB_OK;
}

dnb_status dnb_comm_connect(dnb_comm comm, const void *handles) {
    Comm *c = static_cast<Comm *>(comm);
    if (!c || !handles) return fail(DNB_ERR_INVALID, "comm_connect: null pointer");
    if (c->connected) return DNB_OK;
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    if (device != c->device) return fail(DNB_ERR_INVALID, "comm_connect: communicator of device %d on device %d",
                                         c->device, device);
    for (int r = 0; r < c->world; ++r) {
        if (r == c->rank) continue;
        cudaIpcMemHandle_t h;
        memcpy(&h, static_cast<const char *>(handles) + 64 * (size_t)r, sizeof(h));
        void *p = nullptr;
        cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
        if (e != cudaSuccess) {
            for (int q = 0; q < r; ++q)
                if (q != c->rank && c->peer[q]) {
                    cudaIpcCloseMemHandle(c->peer[q]);
                    c->peer[q] = nullptr;
                }
            return cuda_fail(e, "comm_connect: cudaIpcOpenMemHandle", __FILE__, __LINE__);
        }
        c->peer[r] = p;
    }
    c->connected = true;
    return DNB_OK;
}

dnb_status dnb_comm_destroy(dnb_comm comm) {
    Comm *c = static_cast<Comm *>(comm);
    if (!c) return DNB_OK;
    DNB_CUDA(cudaDeviceSynchronize());
    for (int r = 0; r < c->world; ++r)
        if (r != c->rank && c->peer[r]) cudaIpcCloseMemHandle(c->peer[r]);
    if (c->local) cudaFree(c->local);
    delete c;
    return DNB_OK;
}

}  // extern "C"
