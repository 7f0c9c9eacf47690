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

// Records a thread-local error message and returns `code`.
int set_error(int code, const char* fmt, ...);

// Cached properties of the current device (nullptr + error set on failure).
const DeviceInfo* device_info();

int dtype_size(int dt);

// Raises the kernel's dynamic shared memory limit once per (kernel, device).
int ensure_smem_attr(const void* fn, uint32_t bytes);

struct Gemv3Plan {
    int rows, mt, upc, tpu, gpk, ug, ksplit;
    int even_k;  // 1: every warp of every K slice owns an even number of k-blocks
    int grid, owned, n_units, ring_slots, slot_bytes, nkbw, p_max, xrow_pitch;
    int64_t total_chunks, ws_bytes;
    uint32_t smem_ring, smem_x, smem_xsum, smem_gamma, smem_part, smem_misc, smem_total;
};

// GEMV (per-warp cp.async weight rings, unit-group slots): rows per launch,
// plan, launch.
int gemv3_rows_per_launch(const bq_gemv_desc* d);
int plan_gemv3(const bq_gemv_desc* d, int rows, Gemv3Plan* pl, int slots = 0);
int gemv3_tile_bytes(int fmt, int gpk);
int gemv3_gpk(const bq_gemv_desc* d);
int launch_gemv3(const bq_gemv_desc* d, const Gemv3Plan& pl, int row0, void* workspace, cudaStream_t stream);

// Tensor-core GEMV (tcgen05, weights read once for 17..128 rows).
struct TcPlan {
    int n_mma, KB, units, C, grid, wst;
    uint32_t w_stage, w_bytes, tx_bytes, sm_x, sm_w, sm_bar, sm_total, red_pitch;
    int64_t xn_off, ws_bytes;
};
bool plan_tc(const bq_gemv_desc* d, TcPlan* pl);
int launch_tc(const bq_gemv_desc* d, const TcPlan& pl, void* workspace, cudaStream_t stream);

// Resident-slice GEMV (1..8 rows, whole weight slice in shared memory before the
// dependent-launch wait, no workspace).
struct LeanPlan {
    int units, grid, upc, tpu, nkw, pitch, rbk;
    int ks;  // K slices per unit (clusters of ks CTAs), 1 = no split
    uint32_t sm_w, sm_sc, sm_x, sm_xs, sm_part, sm_misc, sm_red, sm_bar, sm_total;
};
bool plan_lean(const bq_gemv_desc* d, LeanPlan* pl);
int launch_lean(const bq_gemv_desc* d, const LeanPlan& pl, cudaStream_t stream);

// The no-alloc GEMV's built-in scratch: clear its counters again on the next call on `dev`.
void noalloc_forget(int dev);

}  // namespace bq
