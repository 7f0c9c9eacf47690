// Resident-slice GEMV kernels for int4 weights (tinygemm and plain layouts).
#include "bq_lean_kinst.h"

namespace bq {
const void* lean_kernel_int4(int fmt, int tpu, int upc, int rows, int ks) {
    return fmt == BQ_W_INT4_TINYGEMM ? lean_select<BQ_W_INT4_TINYGEMM>(tpu, upc, rows, ks)
                                     : lean_select<BQ_W_INT4_PLAIN>(tpu, upc, rows, ks);
}
}  // namespace bq
