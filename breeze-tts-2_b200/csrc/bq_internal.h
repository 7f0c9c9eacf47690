// Internal declarations shared by the host launchers and the kernels.
#pragma once

#include <cuda.h>
#include <stdint.h>

#include "breeze_b200.h"

#define BQ_DEVERR_WAIT_TIMEOUT_BIT 1u
#define BQ_DEVERR_POSITION_BIT 2u

namespace bq {

constexpr int kKB = 128;          // k per chunk (one k-block)
constexpr int kBoxBytes = 1024;   // one weight tile per k-block: 16 rows x 64 B, or 2 x 8-row tinygemm tiles of 512 B
// Arrival counters live in a fixed region at the start of the workspace, so
// calls of different shapes sharing one workspace never overlap a counter
// with another call's partial sums.
constexpr int kMaxUnits = 65536;
constexpr int64_t kCounterBytes = int64_t(kMaxUnits) * 4;

}  // namespace bq
