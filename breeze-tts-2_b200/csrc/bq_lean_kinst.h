// Kernel-table helper of the resident-slice GEMV (one translation unit per
// weight family keeps compile times short).
#pragma once

#include "bq_lean.cuh"

namespace bq {

template <int FMT>
const void* lean_select(int tpu, int upc) {
    if (tpu == 2) {
        if (upc <= 1) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 1>);
        if (upc <= 2) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 2>);
        return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 4>);
    }
    if (upc <= 1) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 1>);
    if (upc <= 2) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 2>);
    return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 4>);
}

}  // namespace bq
