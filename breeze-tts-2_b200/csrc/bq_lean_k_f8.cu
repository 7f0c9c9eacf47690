// Resident-slice GEMV kernels for 8-bit weights (fp8 e4m3 and int8).
#include "bq_lean_kinst.h"

namespace bq {
const void* lean_kernel_f8(int fmt, int tpu, int upc, int rows, int ks) {
    return fmt == BQ_W_FP8_E4M3 ? lean_select<BQ_W_FP8_E4M3>(tpu, upc, rows, ks)
                                : lean_select<BQ_W_INT8>(tpu, upc, rows, ks);
}
}  // namespace bq
