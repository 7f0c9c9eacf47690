// Internal declarations shared by the host launchers and the kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "breeze_b200.h"

#define BQ_DEVERR_WAIT_TIMEOUT_BIT 1u
#define BQ_DEVERR_POSITION_BIT 2u

namespace bq {

constexpr int kKB = 128;          // k per chunk (one k-block)
constexpr int kTileRows = 16;     // output rows per MMA tile (A operand rows)
constexpr int kUnitRows = 32;     // two tiles per unit
constexpr int kBoxBytes = 1024;   // one TMA box: 16 rows x 64 B, or 2 nTiles x 512 B
constexpr int kMaxMT = 2;         // activation rows per launch = 8 * MT
constexpr int kWarpsPerCta = 8;   // stream-K workers per CTA
// Arrival counters live in a fixed region at the start of the workspace, so
// calls of different shapes sharing one workspace never overlap a counter
// with another call's partial sums.
constexpr int kMaxUnits = 65536;
constexpr int64_t kCounterBytes = int64_t(kMaxUnits) * 4;

// Everything the GEMV kernel needs besides the tensor maps.
struct GemvParams {
    int32_t M, N, K;
    int32_t n_units;      // 32-row units (SILU: 16 gate + 16 up rows)
    int32_t kb_count;     // K / 128
    int32_t epi;
    int32_t group;        // int4 group size
    int32_t x_dtype, out_dtype, res_dtype;
    uint32_t flags;
    float eps;
    int32_t n_half;       // SILU: N / 2
    int32_t workers;      // stream-K workers actually used (<= grid * warps)
    int64_t total_chunks; // n_units * kb_count
    int32_t p_max;        // partial slots per unit
    int32_t ring_slots;   // TMA ring depth per warp
    int32_t slot_bytes;   // bytes per ring slot
    int32_t xfrag_kb;     // k-blocks of staged activations per CTA
    const void* x;
    int64_t ldx;
    const void* gamma;
    const void* scale;    // fp8 / int8 per-row scale (fp32 [N])
    const void* bias;
    const void* residual;
    int64_t ldr;
    void* out;
    int64_t ldo;
    unsigned int* counters;
    float* partials;
};

}  // namespace bq
