// Resident-slice GEMV kernels for bf16 weights.
#include "bq_lean_kinst.h"

namespace bq {
const void* lean_kernel_bf16(int tpu, int upc, int rows, int ks) {
    return lean_select<BQ_W_BF16>(tpu, upc, rows, ks);
}
}  // namespace bq
