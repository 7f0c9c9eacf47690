// Host-side helpers shared by the launchers (not part of the public ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "bq_internal.h"

namespace bq {

struct DeviceInfo {
    int device;
    int sm_count;
    int smem_optin;  // max dynamic shared memory per block (opt-in)
    int major, minor;
};

struct GemvPlan {
    int mt, gpk;
    int grid, workers, ring_slots, slot_bytes, xfrag_kb, p_max, n_units;
    int64_t total_chunks;
    uint32_t smem;
    int64_t counters_bytes, partials_bytes;
};

// Records a thread-local error message and returns `code`.
int set_error(int code, const char* fmt, ...);

// Cached properties of the current device (nullptr + error set on failure).
const DeviceInfo* device_info();

int dtype_size(int dt);

// Raises the kernel's dynamic shared memory limit once per (kernel, device).
int ensure_smem_attr(const void* fn, uint32_t bytes);

// Builds the TMA descriptors for the weight tensor and, for int4, the
// [K/g, N, 2] scale/zero tensor.
int encode_weight_maps(const bq_gemv_desc* d, CUtensorMap* tm_w, CUtensorMap* tm_sz);

int plan_gemv(const bq_gemv_desc* d, int rows, GemvPlan* pl);
int launch_gemv(const bq_gemv_desc* d, const GemvPlan& pl, int row0, int rows, void* workspace,
                cudaStream_t stream);

}  // namespace bq
