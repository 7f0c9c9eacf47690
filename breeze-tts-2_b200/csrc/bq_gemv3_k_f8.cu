// v3 GEMV kernel variants: 8-bit weights (fp8 e4m3 and int8).
#include "bq_gemv3_kinst.h"

namespace bq {
const void* gemv3_kernel_f8(int fmt, int mt, int tpu, bool rect, bool even) {
    if (fmt == BQ_W_FP8_E4M3) return k3_select<BQ_W_FP8_E4M3, 1>(mt, tpu, rect, even);
    return k3_select<BQ_W_INT8, 1>(mt, tpu, rect, even);
}
}  // namespace bq
