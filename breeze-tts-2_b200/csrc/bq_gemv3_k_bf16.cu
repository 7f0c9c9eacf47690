// v3 GEMV kernel variants: bf16 weights.
#include "bq_gemv3_kinst.h"

namespace bq {
const void* gemv3_kernel_bf16(int mt, int tpu, bool rect, bool even) { return k3_select<BQ_W_BF16, 1>(mt, tpu, rect, even); }
}  // namespace bq
