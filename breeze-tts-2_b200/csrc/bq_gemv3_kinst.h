// Instantiation helper for the v3 GEMV kernel: one dispatcher per format file
// so the kernel variants compile in parallel.
#pragma once
#include "bq_gemv3.cuh"

namespace bq {

template <int FMT, int MT, int TPU, int GPK, bool RECT = false>
inline const void* k3() {
    return reinterpret_cast<const void*>(&gemv3_kernel<FMT, MT, TPU, GPK, RECT>);
}

// rect (K split across CTAs) exists for one-tile units only
template <int FMT, int GPK>
inline const void* k3_select(int mt, int tpu, bool rect) {
    if (rect) return tpu != 1 ? nullptr : (mt == 1 ? k3<FMT, 1, 1, GPK, true>() : k3<FMT, 2, 1, GPK, true>());
    if (mt == 1) return tpu == 1 ? k3<FMT, 1, 1, GPK>() : k3<FMT, 1, 2, GPK>();
    return tpu == 1 ? k3<FMT, 2, 1, GPK>() : k3<FMT, 2, 2, GPK>();
}

template <int FMT, int GPK>
inline const void* kc_select(int mt) {
    return mt == 1 ? reinterpret_cast<const void*>(&gemv_chain_kernel<FMT, 1, GPK>)
                   : reinterpret_cast<const void*>(&gemv_chain_kernel<FMT, 2, GPK>);
}

const void* gemv_chain_kernel_int4(int fmt, int mt, int gpk);
const void* gemv_chain_kernel_f8(int fmt, int mt);
const void* gemv_chain_kernel_bf16(int mt);
const void* gemv3_kernel_int4(int fmt, int mt, int tpu, int gpk, bool rect);
const void* gemv3_kernel_f8(int fmt, int mt, int tpu, bool rect);
const void* gemv3_kernel_bf16(int mt, int tpu, bool rect);

}  // namespace bq
