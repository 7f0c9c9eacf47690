// bq_gemv_noalloc: the stream-K GEMV for callers that cannot allocate device
// memory.
//
// Some hosts of this library are not allowed to call cudaMalloc at all: a
// decode loop pinned to a fixed VRAM budget (small cards run the model with a
// hard per-process memory cap), a plugin whose host application owns every
// device allocation through its own allocator, or a real-time audio thread
// that must not take the driver's allocation lock or the implicit device
// synchronization of cudaMalloc/cudaFree. bq_gemv needs a caller-provided
// workspace for its split-K partial sums and arrival counters; this entry
// point instead uses one fixed scratch array that lives in the library's
// device image, so the caller passes only inputs and outputs.
//
// Limits and sharing rules:
//  * The scratch holds kNoAllocScratchBytes (4 MiB) per device: the arrival
//    counters (up to 65536 units of 32 output rows) plus up to 3.75 MiB of
//    partial sums. A shape that needs more is rejected with BQ_ERR_WORKSPACE
//    and nothing is launched. Every GPU that loads the library holds these
//    4 MiB until the process exits.
//  * All calls on a device share the one array and it keeps whatever the
//    last call left there. The counters must start at zero: the first call on
//    a device clears them, and every call that completes leaves them at zero
//    again. Calls whose kernels can overlap on the GPU (different streams with
//    no ordering between them) race on the array and produce wrong results;
//    serialize them on one stream.
//  * The first call on each device does a one-time set-up (looks up the
//    device address of the array and clears the counters, a blocking
//    operation). Make that first call before any stream capture.
//  * No cudaMalloc, cudaFree or allocating library routine is called.
#include <cuda_runtime.h>

#include <mutex>

#include "bq_host.h"

namespace bq {

constexpr int64_t kNoAllocScratchBytes = int64_t(4) << 20;

// The scratch itself. In host code this name is only a handle for the
// runtime; the device address comes from cudaGetSymbolAddress below.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_na_mu;
void* g_na_ptr[128] = {};
}  // namespace

// Device address of the scratch on the current device (set up once per device).
static int noalloc_scratch(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
    if (dev < 0 || dev >= 128) return set_error(BQ_ERR_CUDA, "device ordinal %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_na_mu);
    if (!g_na_ptr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess)
            return set_error(BQ_ERR_CUDA, "cudaGetSymbolAddress(no-alloc scratch): %s", cudaGetErrorString(e));
        e = cudaMemset(p, 0, size_t(kCounterBytes));
        if (e == cudaSuccess) e = cudaDeviceSynchronize();
        if (e != cudaSuccess)
            return set_error(BQ_ERR_CUDA, "clearing the no-alloc scratch counters: %s", cudaGetErrorString(e));
        g_na_ptr[dev] = p;
    }
    *out = g_na_ptr[dev];
    return BQ_OK;
}

int validate_gemv(const bq_gemv_desc* d);

}  // namespace bq

using namespace bq;

extern "C" int32_t bq_gemv_noalloc(const bq_gemv_desc* desc, void* stream) {
    int rc = validate_gemv(desc);
    if (rc) return rc;
    const DeviceInfo* di = device_info();
    if (!di) return BQ_ERR_CUDA;
    if (di->major != 10)
        return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", di->major, di->minor);
    // Check every row block against the scratch size before launching anything.
    constexpr int kRows = 16;
    for (int row0 = 0; row0 < desc->M; row0 += kRows) {
        const int rows = desc->M - row0 < kRows ? desc->M - row0 : kRows;
        GemvPlan pl;
        rc = plan_gemv(desc, rows, &pl);
        if (rc) return rc;
        const int64_t need = pl.counters_bytes + pl.partials_bytes;
        if (need > kNoAllocScratchBytes)
            return set_error(BQ_ERR_WORKSPACE,
                             "bq_gemv_noalloc: this shape needs %lld bytes of scratch, the fixed array holds %lld "
                             "(use bq_gemv with a workspace)",
                             (long long)need, (long long)kNoAllocScratchBytes);
    }
    void* scratch = nullptr;
    rc = noalloc_scratch(&scratch);
    if (rc) return rc;
    for (int row0 = 0; row0 < desc->M; row0 += kRows) {
        const int rows = desc->M - row0 < kRows ? desc->M - row0 : kRows;
        GemvPlan pl;
        rc = plan_gemv(desc, rows, &pl);
        if (rc) return rc;
        rc = launch_gemv(desc, pl, row0, rows, scratch, static_cast<cudaStream_t>(stream));
        if (rc) return rc;
    }
    return BQ_OK;
}
