// Kernel-table helper of the resident-slice GEMV (one translation unit per
// weight family keeps compile times short).
#pragma once

#include "bq_lean.cuh"

namespace bq {

template <int FMT, int MR>
const void* lean_select_m(int tpu, int upc) {
    if (tpu == 2) {
        if (upc <= 1) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 1, MR>);
        if (upc <= 2) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 2, MR>);
        if (upc <= 3) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 3, MR>);
        return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 2, 4, MR>);
    }
    if (upc <= 1) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 1, MR>);
    if (upc <= 2) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 2, MR>);
    if (upc <= 3) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 3, MR>);
    return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 4, MR>);
}

// rows: 1 or 2; ks: 1, or 2 (K split across a cluster of two CTAs per unit: one
// unit per CTA, no SiLU*up)
template <int FMT>
const void* lean_select(int tpu, int upc, int rows, int ks) {
    if (ks == 2) {
        if (tpu != 1 || upc != 1) return nullptr;
        if (rows == 1) return reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 1, 1, 2>);
        return rows == 2 ? reinterpret_cast<const void*>(&gemv_lean_kernel<FMT, 1, 1, 2, 2>) : nullptr;
    }
    if (ks != 1) return nullptr;
    if (rows == 1) return lean_select_m<FMT, 1>(tpu, upc);
    return rows == 2 ? lean_select_m<FMT, 2>(tpu, upc) : nullptr;
}

}  // namespace bq
