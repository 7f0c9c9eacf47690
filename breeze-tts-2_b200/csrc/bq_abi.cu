// C ABI entry points (include/breeze_b200.h), argument validation, error
// reporting and the device property cache.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <vector>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

// Device error word, one per device: bounded waits that give up set bits here
// (read and cleared through bq_device_status / bq_device_status_clear).
__device__ unsigned int g_device_error = 0;

namespace {
thread_local char g_err[512] = "no error";
std::mutex g_mu;
std::vector<DeviceInfo> g_dev;                         // indexed by device ordinal
std::vector<std::pair<const void*, int>> g_smem_attr;  // (kernel, device) raised
}  // namespace

int set_error(int code, const char* fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof(g_err), fmt, ap);
    va_end(ap);
    return code;
}

const DeviceInfo* device_info() {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        set_error(BQ_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_mu);
    if (int(g_dev.size()) <= dev) g_dev.resize(dev + 1, DeviceInfo{-1, 0, 0, 0, 0});
    DeviceInfo& d = g_dev[dev];
    if (d.device < 0) {
        DeviceInfo n{dev, 0, 0, 0, 0};
        if (cudaDeviceGetAttribute(&n.sm_count, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
            cudaDeviceGetAttribute(&n.minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess) {
            set_error(BQ_ERR_CUDA, "cudaDeviceGetAttribute failed on device %d", dev);
            return nullptr;
        }
        d = n;
    }
    return &d;
}

int dtype_size(int dt) { return dt == BQ_DT_F32 ? 4 : 2; }

int ensure_smem_attr(const void* fn, uint32_t bytes) {
    int dev = 0;
    cudaGetDevice(&dev);
    {
        std::lock_guard<std::mutex> lk(g_mu);
        for (auto& kv : g_smem_attr)
            if (kv.first == fn && kv.second == dev) return BQ_OK;
    }
    const DeviceInfo* di = device_info();
    if (!di) return BQ_ERR_CUDA;
    cudaFuncAttributes fa;
    cudaError_t e = cudaFuncGetAttributes(&fa, fn);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "cudaFuncGetAttributes: %s", cudaGetErrorString(e));
    // static shared memory counts against the same opt-in limit
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, di->smem_optin - int(fa.sharedSizeBytes));
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "cudaFuncSetAttribute: %s", cudaGetErrorString(e));
    (void)bytes;
    std::lock_guard<std::mutex> lk(g_mu);
    g_smem_attr.emplace_back(fn, dev);
    return BQ_OK;
}

// ---- validation -------------------------------------------------------------
static bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

int validate_gemv(const bq_gemv_desc* d) {
    if (!d) return set_error(BQ_ERR_INVALID_ARG, "desc is NULL");
    if (d->M < 1 || d->N < 1 || d->K < 1)
        return set_error(BQ_ERR_SHAPE, "M, N, K must be positive (got %d, %d, %d)", d->M, d->N, d->K);
    if (d->K % 128) return set_error(BQ_ERR_SHAPE, "K=%d must be a multiple of 128", d->K);
    if (d->wfmt < BQ_W_BF16 || d->wfmt > BQ_W_INT8) return set_error(BQ_ERR_FORMAT, "unknown weight format %d", d->wfmt);
    if (d->epilogue < BQ_EPI_NONE || d->epilogue > BQ_EPI_ADD_RESIDUAL)
        return set_error(BQ_ERR_INVALID_ARG, "unknown epilogue %d", d->epilogue);
    for (int dt : {d->x_dtype, d->out_dtype, d->res_dtype})
        if (dt < BQ_DT_BF16 || dt > BQ_DT_F32) return set_error(BQ_ERR_INVALID_ARG, "unknown dtype %d", dt);
    if (!d->x || !d->w || !d->out) return set_error(BQ_ERR_INVALID_ARG, "x, w and out must be non-NULL");
    if (d->ldx < d->K) return set_error(BQ_ERR_SHAPE, "ldx=%lld < K=%d", (long long)d->ldx, d->K);
    const int n_out = d->epilogue == BQ_EPI_SILU_MUL ? d->N / 2 : d->N;
    if (d->ldo < n_out) return set_error(BQ_ERR_SHAPE, "ldo=%lld < output width %d", (long long)d->ldo, n_out);
    if (d->epilogue == BQ_EPI_SILU_MUL && (d->N % 2))
        return set_error(BQ_ERR_SHAPE, "SiLU*up epilogue needs an even N (got %d)", d->N);
    if (d->epilogue == BQ_EPI_ADD_RESIDUAL) {
        if (!d->residual) return set_error(BQ_ERR_INVALID_ARG, "residual epilogue without a residual");
        if (d->ldr < n_out) return set_error(BQ_ERR_SHAPE, "ldr=%lld < output width %d", (long long)d->ldr, n_out);
    }
    if (!aligned16(d->w)) return set_error(BQ_ERR_ALIGN, "weight pointer must be 16-byte aligned");
    const bool int4 = d->wfmt == BQ_W_INT4_TINYGEMM || d->wfmt == BQ_W_INT4_PLAIN;
    if (int4 || d->wfmt == BQ_W_FP8_E4M3 || d->wfmt == BQ_W_INT8) {
        if (!d->scale) return set_error(BQ_ERR_INVALID_ARG, "this weight format needs a scale tensor");
    }
    if (int4) {
        if (!aligned16(d->scale)) return set_error(BQ_ERR_ALIGN, "scale/zero tensor must be 16-byte aligned");
        if (d->N % 8) return set_error(BQ_ERR_SHAPE, "int4 weights need N %% 8 == 0 (got %d)", d->N);
        if (d->epilogue == BQ_EPI_SILU_MUL && ((d->N / 2) % 8))
            return set_error(BQ_ERR_SHAPE, "int4 SiLU*up needs (N/2) %% 8 == 0 (got N=%d)", d->N);
        if (d->wfmt == BQ_W_INT4_TINYGEMM) {
            if (d->group != 32 && d->group != 64 && d->group != 128 && d->group != 256)
                return set_error(BQ_ERR_SHAPE, "tinygemm int4 group must be 32, 64, 128 or 256 (got %d)", d->group);
            if (d->K % d->group) return set_error(BQ_ERR_SHAPE, "K=%d not divisible by group %d", d->K, d->group);
        } else if (d->group != 128) {
            return set_error(BQ_ERR_SHAPE, "plain int4 layout uses group 128 (got %d)", d->group);
        }
    }
    return BQ_OK;
}

}  // namespace bq

using namespace bq;


extern "C" {

int32_t bq_version(void) { return BQ_VERSION; }

const char* bq_last_error_string(void) { return g_err; }

int32_t bq_device_status(int32_t device, uint32_t* bits) {
    if (!bits) return set_error(BQ_ERR_INVALID_ARG, "bits is NULL");
    int prev = 0;
    cudaGetDevice(&prev);
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMemcpyFromSymbol(bits, g_device_error, sizeof(uint32_t));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "reading device status: %s", cudaGetErrorString(e));
    return BQ_OK;
}

int32_t bq_device_status_clear(int32_t device) {
    int prev = 0;
    cudaGetDevice(&prev);
    const uint32_t zero = 0;
    cudaError_t e = cudaSetDevice(device);
    if (e == cudaSuccess) e = cudaMemcpyToSymbol(g_device_error, &zero, sizeof(uint32_t));
    cudaSetDevice(prev);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "clearing device status: %s", cudaGetErrorString(e));
    noalloc_forget(device);  // a timed-out kernel may have left the built-in scratch's counters set
    return BQ_OK;
}

int32_t bq_gemv_workspace_bytes(const bq_gemv_desc* desc, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    int rc = validate_gemv(desc);
    if (rc) return rc;
    TcPlan tp;
    if (plan_tc(desc, &tp)) {
        *bytes = size_t(tp.ws_bytes);
        return BQ_OK;
    }
    LeanPlan lp;
    if (plan_lean(desc, &lp)) {
        *bytes = 0;
        return BQ_OK;
    }
    const int step = gemv3_rows_per_launch(desc);
    int64_t need = 0;
    for (int row0 = 0; row0 < desc->M; row0 += step) {
        Gemv3Plan pl;
        rc = plan_gemv3(desc, std::min(step, desc->M - row0), &pl);
        if (rc) return rc;
        need = std::max(need, pl.ws_bytes);
    }
    *bytes = size_t(need);
    return BQ_OK;
}

int32_t bq_gemv(const bq_gemv_desc* desc, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate_gemv(desc);
    if (rc) return rc;
    if (desc->gamma && (reinterpret_cast<uintptr_t>(desc->gamma) & 15))
        return set_error(BQ_ERR_ALIGN, "gamma must be 16-byte aligned");
    const DeviceInfo* di = device_info();
    if (!di) return BQ_ERR_CUDA;
    if (di->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", di->major, di->minor);
    TcPlan tp;
    if (plan_tc(desc, &tp)) {
        if (tp.ws_bytes > 0 && (!workspace || int64_t(workspace_bytes) < tp.ws_bytes))
            return set_error(BQ_ERR_WORKSPACE, "workspace of %zu bytes given, %lld needed", workspace_bytes,
                             (long long)tp.ws_bytes);
        if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
            return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
        return launch_tc(desc, tp, workspace, static_cast<cudaStream_t>(stream));
    }
    LeanPlan lp;
    if (plan_lean(desc, &lp)) return launch_lean(desc, lp, static_cast<cudaStream_t>(stream));
    const int step = gemv3_rows_per_launch(desc);
    for (int row0 = 0; row0 < desc->M; row0 += step) {
        Gemv3Plan pl;
        rc = plan_gemv3(desc, std::min(step, desc->M - row0), &pl);
        if (rc) return rc;
        if (pl.ws_bytes > 0) {
            if (!workspace || int64_t(workspace_bytes) < pl.ws_bytes)
                return set_error(BQ_ERR_WORKSPACE, "workspace of %zu bytes given, %lld needed", workspace_bytes,
                                 (long long)pl.ws_bytes);
            if ((reinterpret_cast<uintptr_t>(workspace) & 255) != 0)
                return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
        }
        rc = launch_gemv3(desc, pl, row0, workspace, static_cast<cudaStream_t>(stream));
        if (rc) return rc;
    }
    return BQ_OK;
}

int32_t bq_gemv_host_io(const bq_gemv_desc* desc, const void* x_host, void* out_host, void* workspace,
                        size_t workspace_bytes, void* stream) {
    int rc = validate_gemv(desc);
    if (rc) return rc;
    if (!x_host || !out_host) return set_error(BQ_ERR_INVALID_ARG, "x_host and out_host must be non-NULL");
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const size_t xs = size_t(dtype_size(desc->x_dtype)), os = size_t(dtype_size(desc->out_dtype));
    const size_t n_out = size_t(desc->epilogue == BQ_EPI_SILU_MUL ? desc->N / 2 : desc->N);
    // dense host rows into the (possibly strided) device activations
    cudaError_t e = cudaMemcpy2DAsync(const_cast<void*>(desc->x), size_t(desc->ldx) * xs, x_host, size_t(desc->K) * xs,
                                      size_t(desc->K) * xs, size_t(desc->M), cudaMemcpyHostToDevice, st);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "input copy failed: %s", cudaGetErrorString(e));
    rc = bq_gemv(desc, workspace, workspace_bytes, stream);
    if (rc) return rc;
    e = cudaMemcpy2DAsync(out_host, n_out * os, desc->out, size_t(desc->ldo) * os, n_out * os, size_t(desc->M),
                          cudaMemcpyDeviceToHost, st);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "output copy failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
