// bq_gemv_noalloc: bq_gemv for callers that cannot allocate device memory.
//
// Some hosts of this library are not allowed to call cudaMalloc at all: a
// decode loop pinned to a fixed VRAM budget (small cards run the model with a
// hard per-process memory cap), a plugin whose host application owns every
// device allocation through its own allocator, or a real-time audio thread
// that must not take the driver's allocation lock or the implicit device
// synchronization of cudaMalloc/cudaFree. bq_gemv needs a caller-provided
// workspace for its split-K partial sums and arrival counters; this entry
// point runs the same kernel and plan with one fixed scratch array that lives
// in the library's device image, so the caller passes only inputs and outputs.
//
// Limits and sharing rules:
//  * The scratch holds kNoAllocScratchBytes (4 MiB) per device: the arrival
//    counters (256 KiB, one word per unit) plus up to 3.75 MiB of partial
//    sums. A shape that needs more (bq_gemv_workspace_bytes) is rejected with
//    BQ_ERR_WORKSPACE and nothing is launched. Every GPU that loads the
//    library holds these 4 MiB until the process exits.
//  * All calls on a device share the one array, which keeps whatever the last
//    call left there. The counters must start at zero: the first call on a
//    device clears them. The kernel has no waits -- the last CTA to reach a
//    unit sums its pieces and resets the unit's counter -- so every launch
//    that runs to completion leaves them at zero again. Calls whose kernels
//    can overlap on the GPU (different streams with no ordering between them)
//    race on the array and produce wrong results; serialize them on one
//    stream.
//  * The array's device address is looked up on every call (no
//    synchronization). The first call on each device, and the first call
//    after the library's device image was reloaded (a cudaDeviceReset),
//    clears the counters with a blocking memset: make that call before any
//    stream capture.
//  * A kernel whose bounded wait ran out (BQ_DEVERR_WAIT_TIMEOUT) may leave
//    counters non-zero. bq_device_status_clear on that device marks the
//    array for clearing again, so the next call here starts from zeroed
//    counters (the same blocking memset: outside stream capture).
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>

#include "bq_host.h"

namespace bq {

constexpr int64_t kNoAllocScratchBytes = int64_t(4) << 20;
static_assert(kNoAllocScratchBytes > kCounterBytes, "scratch must hold the arrival counters");

// The scratch itself. In host code this name is only a handle for the
// runtime; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
constexpr int kMaxDevices = 128;
std::mutex g_na_mu;
void* g_na_cleared[kMaxDevices] = {};  // per device: the address whose counters were cleared
}  // namespace

// Device address of the scratch on the current device, counters cleared once
// per (device, address).
static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= kMaxDevices) return set_error(BQ_ERR_CUDA, "device ordinal %d out of range", dev);
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
        return set_error(BQ_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (g_na_cleared[dev] != p) {
        e = cudaMemset(p, 0, size_t(kCounterBytes));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess)
            return set_error(BQ_ERR_CUDA, "clearing the no-alloc scratch counters: %s", cudaGetErrorString(e));
        g_na_cleared[dev] = p;
    }
    *out = p;
    return BQ_OK;
}

// Called by bq_device_status_clear: the next call on `dev` clears the
// counters again (after a timeout they may not have returned to zero).
void noalloc_forget(int dev) {
    if (dev < 0 || dev >= kMaxDevices) return;
    std::lock_guard<std::mutex> lk(g_na_mu);
    g_na_cleared[dev] = nullptr;
}

}  // namespace bq

using namespace bq;

extern "C" int32_t bq_gemv_noalloc(const bq_gemv_desc* desc, void* stream) {
    size_t need = 0;
    int rc = bq_gemv_workspace_bytes(desc, &need);  // validates the descriptor, plans every row block
    if (rc) return rc;
    bq_gemv_desc rows16;
    if (int64_t(need) > kNoAllocScratchBytes && !(desc->flags & BQ_FLAG_NO_TC)) {
        // the tensor-core kernel's per-CTA pieces do not fit: the row-block kernel needs less
        rows16 = *desc;
        rows16.flags |= BQ_FLAG_NO_TC;
        rc = bq_gemv_workspace_bytes(&rows16, &need);
        if (rc) return rc;
        desc = &rows16;
    }
    if (int64_t(need) > kNoAllocScratchBytes)
        return set_error(BQ_ERR_WORKSPACE,
                         "bq_gemv_noalloc: this shape needs %zu bytes of scratch, the fixed array holds %lld "
                         "(use bq_gemv with a workspace)",
                         need, (long long)kNoAllocScratchBytes);
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    return bq_gemv(desc, scratch, size_t(kNoAllocScratchBytes), stream);
}
