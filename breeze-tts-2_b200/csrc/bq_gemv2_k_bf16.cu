// v2 GEMV kernel variants: bf16 weights.
#include "bq_gemv2_kinst.h"

namespace bq {
const void* gemv2_kernel_bf16(int mt, int tpu) { return k2_select<BQ_W_BF16, 1>(mt, tpu); }
}  // namespace bq
