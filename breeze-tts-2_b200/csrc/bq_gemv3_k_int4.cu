// v3 GEMV kernel variants: int4 weights (tinygemm and plain layouts).
#include "bq_gemv3_kinst.h"

namespace bq {
const void* gemv3_kernel_int4(int fmt, int mt, int tpu, int gpk, bool rect, bool even) {
    if (fmt == BQ_W_INT4_PLAIN) return gpk == 1 ? k3_select<BQ_W_INT4_PLAIN, 1>(mt, tpu, rect, even) : nullptr;
    if (gpk == 1) return k3_select<BQ_W_INT4_TINYGEMM, 1>(mt, tpu, rect, even);
    if (gpk == 2) return k3_select<BQ_W_INT4_TINYGEMM, 2>(mt, tpu, rect, even);
    if (gpk == 4) return k3_select<BQ_W_INT4_TINYGEMM, 4>(mt, tpu, rect, even);
    return nullptr;
}
}  // namespace bq
