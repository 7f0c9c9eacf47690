// Instantiation helper for the v3 GEMV kernel: one dispatcher per format file
// so the kernel variants compile in parallel.
#pragma once
#include "bq_gemv3.cuh"

namespace bq {

template <int FMT, int MT, int TPU, int GPK, bool RECT = false, bool EVEN = false>
inline const void* k3() {
    return reinterpret_cast<const void*>(&gemv3_kernel<FMT, MT, TPU, GPK, RECT, EVEN>);
}

// one-row kernels: the EVEN variant when every warp's k-block count is even
template <int FMT, int TPU, int GPK, bool RECT>
inline const void* k3_mt1(bool even) {
    return even ? k3<FMT, 1, TPU, GPK, RECT, true>() : k3<FMT, 1, TPU, GPK, RECT, false>();
}

// rect (K split across CTAs) exists for one-tile units only; EVEN matters for
// one-row kernels only (one k-block per slot otherwise)
template <int FMT, int GPK>
inline const void* k3_select(int mt, int tpu, bool rect, bool even) {
    if (rect) return tpu != 1 ? nullptr : (mt == 1 ? k3_mt1<FMT, 1, GPK, true>(even) : k3<FMT, 2, 1, GPK, true>());
    if (mt == 1) return tpu == 1 ? k3_mt1<FMT, 1, GPK, false>(even) : k3_mt1<FMT, 2, GPK, false>(even);
    return tpu == 1 ? k3<FMT, 2, 1, GPK>() : k3<FMT, 2, 2, GPK>();
}

const void* gemv3_kernel_int4(int fmt, int mt, int tpu, int gpk, bool rect, bool even);
const void* gemv3_kernel_f8(int fmt, int mt, int tpu, bool rect, bool even);
const void* gemv3_kernel_bf16(int mt, int tpu, bool rect, bool even);

}  // namespace bq
