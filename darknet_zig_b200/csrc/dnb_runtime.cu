// Device, memory and error plumbing of libdnb200: the replacement for the reference's
// vendor shim (src/cuda/cuda.zig:248-339) and gpu.zig's init/alloc/push/pull/sync
// (src/gpu.zig:259-410).
#include <stdarg.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <map>
#include <mutex>
#include <utility>

#include "dnb_common.cuh"

namespace dnb {

namespace {

thread_local char g_detail[512] = "";
std::mutex g_mu;
DeviceState g_dev[kMaxDevices];
std::map<std::pair<int, cudaStream_t>, Workspace *> g_ws;
std::atomic<unsigned long long> g_launches{0};
bool g_sync_after_launch = false;
unsigned long long g_wait_limit_ns = 2000ull * 1000ull * 1000ull;  // 2 s

dnb_status init_device(int device) {
    if (device < 0 || device >= kMaxDevices) return fail(DNB_ERR_INVALID, "device index %d out of range", device);
    DeviceState &ds = g_dev[device];
    if (ds.device == device) return DNB_OK;
    DNB_CUDA(cudaSetDevice(device));
    DNB_CUDA(cudaDeviceGetAttribute(&ds.sm_count, cudaDevAttrMultiProcessorCount, device));
    DNB_CUDA(cudaDeviceGetAttribute(&ds.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, device));
    DNB_CUDA(cudaDeviceGetAttribute(&ds.smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device));
    DNB_CUDA(cudaDeviceGetAttribute(&ds.smem_reserved, cudaDevAttrReservedSharedMemoryPerBlock, device));
    unsigned *words = nullptr;
    DNB_CUDA(cudaMalloc(&words, 2 * sizeof(unsigned)));
    DNB_CUDA(cudaMemset(words, 0, 2 * sizeof(unsigned)));
    ds.error_word = words;
    ds.abort_flag = words + 1;
    ds.device = device;
    return DNB_OK;
}

}  // namespace

dnb_status fail(dnb_status s, const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_detail, sizeof(g_detail), fmt, ap);
    va_end(ap);
    return s;
}

dnb_status cuda_fail(cudaError_t e, const char *what, const char *file, int line) {
    const char *base = strrchr(file, '/');
    return fail(e == cudaErrorMemoryAllocation ? DNB_ERR_NO_MEMORY : DNB_ERR_CUDA, "%s failed: %s (%s) at %s:%d",
                what, cudaGetErrorName(e), cudaGetErrorString(e), base ? base + 1 : file, line);
}

dnb_status current_device(DeviceState **out) {
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    std::lock_guard<std::mutex> lock(g_mu);
    DNB_TRY(init_device(device));
    *out = &g_dev[device];
    return DNB_OK;
}

dnb_status workspace(cudaStream_t stream, size_t scratch_bytes, Workspace **out, size_t rec_words) {
    int device = 0;
    DNB_CUDA(cudaGetDevice(&device));
    std::lock_guard<std::mutex> lock(g_mu);
    DNB_TRY(init_device(device));
    Workspace *&ws = g_ws[{device, stream}];
    if (!ws) ws = new Workspace();
    ws->stream = stream;
    const size_t want_sync = kSyncWords;
    bool grow_sync = ws->sync_words < want_sync;
    bool grow_scratch = ws->scratch_bytes < scratch_bytes;
    bool grow_recs = ws->rec_words < rec_words;
    if (grow_sync || grow_scratch || grow_recs) {
        cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
        DNB_CUDA(cudaStreamIsCapturing(stream, &cap));
        if (cap != cudaStreamCaptureStatusNone)
            return fail(DNB_ERR_UNSUPPORTED,
                        "the workspace for this stream must grow (to %zu bytes); run the op once before capture",
                        scratch_bytes);
        DNB_CUDA(cudaStreamSynchronize(stream));
    }
    if (grow_sync) {
        if (ws->sync) DNB_CUDA(cudaFree(ws->sync));
        ws->sync = nullptr;
        DNB_CUDA(cudaMalloc(&ws->sync, want_sync * sizeof(unsigned)));
        DNB_CUDA(cudaMemset(ws->sync, 0, want_sync * sizeof(unsigned)));
        ws->sync_words = want_sync;
    }
    if (grow_scratch) {
        size_t bytes = scratch_bytes < (4u << 20) ? (4u << 20) : scratch_bytes + (scratch_bytes >> 2);
        if (ws->scratch) DNB_CUDA(cudaFree(ws->scratch));
        ws->scratch = nullptr;
        DNB_CUDA(cudaMalloc(&ws->scratch, bytes));
        ws->scratch_bytes = bytes;
    }
    if (grow_recs) {
        // a record word is (tag << 32 | value) and tag 0 is never a launch's: cleared words
        // read as "not written"
        size_t words = rec_words < (1u << 16) ? (1u << 16) : rec_words;
        if (ws->recs) DNB_CUDA(cudaFree(ws->recs));
        ws->recs = nullptr;
        DNB_CUDA(cudaMalloc(&ws->recs, words * sizeof(unsigned long long)));
        DNB_CUDA(cudaMemset(ws->recs, 0, words * sizeof(unsigned long long)));
        ws->rec_words = words;
    }
    *out = ws;
    return DNB_OK;
}

void note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

dnb_status after_launch(cudaStream_t stream, const char *what) {
    note_launch();
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return fail(DNB_ERR_CUDA, "launching %s failed: %s", what, cudaGetErrorString(e));
    if (g_sync_after_launch) {
        e = cudaStreamSynchronize(stream);
        if (e != cudaSuccess) return fail(DNB_ERR_CUDA, "%s faulted: %s", what, cudaGetErrorString(e));
        DeviceState *ds = nullptr;
        DNB_TRY(current_device(&ds));
        unsigned word = 0;
        DNB_CUDA(cudaMemcpy(&word, ds->error_word, sizeof(word), cudaMemcpyDeviceToHost));
        if (word) return fail(DNB_ERR_TIMEOUT, "%s: a device-side wait gave up (error bits 0x%x)", what, word);
    }
    return DNB_OK;
}

unsigned long long wait_limit_ns() { return g_wait_limit_ns; }

bool sync_after_launch() { return g_sync_after_launch; }

}  // namespace dnb

using namespace dnb;

extern "C" {

const char *dnb_error_string(dnb_status s) {
    switch (s) {
    case DNB_OK: return "ok";
    case DNB_ERR_INVALID: return "invalid argument";
    case DNB_ERR_CUDA: return "CUDA error";
    case DNB_ERR_TIMEOUT: return "device-side wait timed out";
    case DNB_ERR_NOT_INIT: return "not initialised";
    case DNB_ERR_UNSUPPORTED: return "unsupported shape or option";
    case DNB_ERR_COMM: return "communicator error";
    case DNB_ERR_NO_MEMORY: return "out of device memory";
    }
    return "unknown status";
}

const char *dnb_last_error_detail(void) { return g_detail; }

dnb_status dnb_init(int device) {
    std::lock_guard<std::mutex> lock(g_mu);
    DNB_TRY(init_device(device));
    DNB_CUDA(cudaSetDevice(device));
    return DNB_OK;
}

dnb_status dnb_device_count(int *count) {
    if (!count) return fail(DNB_ERR_INVALID, "count is null");
    DNB_CUDA(cudaGetDeviceCount(count));
    return DNB_OK;
}

dnb_status dnb_device_name(int device, char *buf, int len) {
    if (!buf || len <= 0) return fail(DNB_ERR_INVALID, "bad name buffer");
    cudaDeviceProp prop;
    DNB_CUDA(cudaGetDeviceProperties(&prop, device));
    snprintf(buf, (size_t)len, "%s", prop.name);
    return DNB_OK;
}

dnb_status dnb_mem_info(size_t *free_bytes, size_t *total_bytes) {
    DNB_CUDA(cudaMemGetInfo(free_bytes, total_bytes));
    return DNB_OK;
}

dnb_status dnb_malloc(void **ptr, size_t bytes) {
    if (!ptr) return fail(DNB_ERR_INVALID, "ptr is null");
    *ptr = nullptr;
    if (bytes == 0) return DNB_OK;
    DNB_CUDA(cudaMalloc(ptr, bytes));
    DNB_CUDA(cudaMemset(*ptr, 0, bytes));
    return DNB_OK;
}

dnb_status dnb_free(void *ptr) {
    if (ptr) DNB_CUDA(cudaFree(ptr));
    return DNB_OK;
}

dnb_status dnb_memset_zero(void *ptr, size_t bytes, dnb_stream stream) {
    if (bytes == 0) return DNB_OK;
    if (!ptr) return fail(DNB_ERR_INVALID, "ptr is null");
    DNB_CUDA(cudaMemsetAsync(ptr, 0, bytes, as_stream(stream)));
    note_launch();
    return DNB_OK;
}

dnb_status dnb_push(void *dst_device, const void *src_host, size_t bytes, dnb_stream stream) {
    if (bytes == 0) return DNB_OK;
    if (!dst_device || !src_host) return fail(DNB_ERR_INVALID, "null pointer");
    DNB_CUDA(cudaMemcpyAsync(dst_device, src_host, bytes, cudaMemcpyHostToDevice, as_stream(stream)));
    return DNB_OK;
}

dnb_status dnb_pull(void *dst_host, const void *src_device, size_t bytes, dnb_stream stream) {
    if (bytes == 0) return DNB_OK;
    if (!dst_host || !src_device) return fail(DNB_ERR_INVALID, "null pointer");
    DNB_CUDA(cudaMemcpyAsync(dst_host, src_device, bytes, cudaMemcpyDeviceToHost, as_stream(stream)));
    return DNB_OK;
}

dnb_status dnb_sync(void) {
    DNB_CUDA(cudaDeviceSynchronize());
    return DNB_OK;
}

dnb_status dnb_stream_sync(dnb_stream stream) {
    DNB_CUDA(cudaStreamSynchronize(as_stream(stream)));
    return DNB_OK;
}

dnb_status dnb_set_sync_after_launch(int on) {
    g_sync_after_launch = on != 0;
    return DNB_OK;
}

dnb_status dnb_check_device_error(void) {
    DeviceState *ds = nullptr;
    DNB_TRY(current_device(&ds));
    DNB_CUDA(cudaDeviceSynchronize());
    unsigned word[2] = {0, 0};
    DNB_CUDA(cudaMemcpy(word, ds->error_word, sizeof(word), cudaMemcpyDeviceToHost));
    if (word[0] == 0 && word[1] == 0) return DNB_OK;
    // A wait gave up: the launch state of every workspace on this device may be mid-launch,
    // so it is reset along with the error word (the epoch restarts, so the records carrying
    // earlier epochs' tags are cleared too).
    DNB_CUDA(cudaMemset(ds->error_word, 0, 2 * sizeof(unsigned)));
    {
        std::lock_guard<std::mutex> lock(g_mu);
        for (auto &kv : g_ws) {
            if (kv.first.first != ds->device) continue;
            if (kv.second->sync) DNB_CUDA(cudaMemset(kv.second->sync, 0, kv.second->sync_words * sizeof(unsigned)));
            if (kv.second->recs)
                DNB_CUDA(cudaMemset(kv.second->recs, 0, kv.second->rec_words * sizeof(unsigned long long)));
        }
    }
    return fail(DNB_ERR_TIMEOUT, "a device-side wait gave up (error bits 0x%x)", word[0]);
}

dnb_status dnb_launch_count(unsigned long long *count) {
    if (!count) return fail(DNB_ERR_INVALID, "launch_count: null pointer");
    *count = g_launches.load(std::memory_order_relaxed);
    return DNB_OK;
}

dnb_status dnb_set_wait_limit_ms(int ms) {
    if (ms <= 0) return fail(DNB_ERR_INVALID, "wait limit must be positive");
    g_wait_limit_ns = (unsigned long long)ms * 1000000ull;
    return DNB_OK;
}

}  // extern "C"
