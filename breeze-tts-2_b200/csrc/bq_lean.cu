// Host planning and launch of the resident-slice GEMV (bq_lean.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "bq_host.h"
#include "bq_lean.cuh"

namespace bq {

const void* lean_kernel_int4(int fmt, int tpu, int upc, int rows, int ks);
const void* lean_kernel_f8(int fmt, int tpu, int upc, int rows, int ks);
const void* lean_kernel_bf16(int tpu, int upc, int rows, int ks);

namespace {
inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

const void* lean_kernel(int fmt, int tpu, int upc, int rows, int ks) {
    if (fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN) return lean_kernel_int4(fmt, tpu, upc, rows, ks);
    if (fmt == BQ_W_FP8_E4M3 || fmt == BQ_W_INT8) return lean_kernel_f8(fmt, tpu, upc, rows, ks);
    if (fmt == BQ_W_BF16) return lean_kernel_bf16(tpu, upc, rows, ks);
    return nullptr;
}
}  // namespace

// The resident-slice kernel applies to one or two bf16 rows (16-byte aligned)
// whose per-warp activation slice fits eight 16-byte chunks per lane, int4
// groups of 128 or 256, at most four units per CTA, and a CTA share that fits
// shared memory. Measured on the 28-layer decode step (per-launch graph, us):
// int4 M = 1 / 2 883 / 922 -> 764 / 901, fp8 877 / 982 -> 760 / 893, int8
// 952 / 1048 -> 807 / 927. At M = 4 and 8 (the row count a compile-time
// parameter there too) it was level or up to 10 % slower than the
// ring-streaming kernel -- its staging and row reductions grow with M -- so
// those keep the ring kernel. BQ_FLAG_RING_KERNEL forces the ring kernel.
// Fewer 16-row units than half the SMs (the depth decoder's down projection:
// 64 units over K = 8192) split K in two across a cluster of two CTAs per unit
// (plain SiLU-free epilogues; the cluster's partial sums meet in distributed
// shared memory), when that gives at least half the SMs a CTA.
bool plan_lean(const bq_gemv_desc* d, LeanPlan* pl) {
    if (d->flags & BQ_FLAG_RING_KERNEL) return false;
    if (d->M < 1 || d->M > 2 || d->x_dtype != BQ_DT_BF16) return false;
    if ((reinterpret_cast<uintptr_t>(d->x) & 15) || (d->ldx % 8) != 0) return false;
    const int fmt = d->wfmt;
    const bool int4 = fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN;
    if (int4 && d->group != 128 && !(fmt == BQ_W_INT4_TINYGEMM && d->group == 256)) return false;
    const int KB = d->K / 128;
    if (KB < 1) return false;
    const DeviceInfo* di = device_info();
    if (!di) return false;
    LeanPlan P{};
    P.tpu = d->epilogue == BQ_EPI_SILU_MUL ? 2 : 1;
    const int n_out = P.tpu == 2 ? d->N / 2 : d->N;
    P.units = (n_out + 15) / 16;
    P.ks = 1;
    if (2 * P.units < di->sm_count) {
        // one unit per CTA, K in two halves of at least eight k-blocks each
        if (P.tpu != 1 || KB % 2 != 0 || KB / 2 < 8) return false;
        P.ks = 2;
        if (P.units * P.ks > di->sm_count || 2 * P.units * P.ks < di->sm_count) return false;
    }
    const int nkw = (KB / P.ks + 7) / 8;
    if (d->M * nkw > 16) return false;
    P.grid = P.ks > 1 ? P.units * P.ks : std::min(di->sm_count, P.units);
    P.upc = P.ks > 1 ? 1 : (P.units + P.grid - 1) / P.grid;
    if (P.upc > 4) return false;
    P.nkw = nkw;
    P.pitch = nkw * 256 + 16;
    P.rbk = fmt == BQ_W_BF16 ? 2 * d->K : (fmt == BQ_W_FP8_E4M3 || fmt == BQ_W_INT8) ? d->K : d->K / 2;
    const int rows_cap = 16 * P.upc;
    uint32_t o = 0;
    P.sm_w = o;  // [half][rows_cap][rbk / ks]: the CTA's rows (K slice) as stored in memory
    o += uint32_t(P.tpu * rows_cap * (P.rbk / P.ks));
    o = align_up(o, 128);
    P.sm_sc = o;  // int4: [kb][half][rows_cap] (scale, zero) words
    if (int4) o += uint32_t(KB * P.tpu * rows_cap * 4);
    o = align_up(o, 128);
    P.sm_x = o;
    o += uint32_t(8 * (d->M * P.pitch + 256));
    o = align_up(o, 16);
    P.sm_xs = o;
    o += uint32_t(8 * nkw * 8 * 4);
    o = align_up(o, 16);
    P.sm_part = o;
    o += uint32_t(P.upc * P.tpu * 8 * 128 * 4);
    o = align_up(o, 16);
    P.sm_misc = o;
    o += 128 * 4;
    o = align_up(o, 16);
    P.sm_red = o;  // K split: [half][16][8] partial sums + [8] sum(x^2)
    if (P.ks > 1) o += uint32_t((P.tpu * 128 + 8) * 4);
    o = align_up(o, 16);
    P.sm_bar = o;
    o += 16;
    P.sm_total = o;
    if (int64_t(P.sm_total) > int64_t(di->smem_optin)) return false;
    if (!lean_kernel(fmt, P.tpu, P.upc, d->M, P.ks)) return false;
    *pl = P;
    return true;
}

int launch_lean(const bq_gemv_desc* d, const LeanPlan& pl, cudaStream_t stream) {
    const void* fn = lean_kernel(d->wfmt, pl.tpu, pl.upc, d->M, pl.ks);
    if (!fn) return set_error(BQ_ERR_FORMAT, "no resident-slice GEMV for format %d", d->wfmt);
    LeanParams p;
    std::memset(&p, 0, sizeof(p));
    p.x = static_cast<const __nv_bfloat16*>(d->x);
    p.ldx = d->ldx;
    p.gamma = static_cast<const __nv_bfloat16*>(d->gamma);
    p.w = d->w;
    p.scale = d->scale;
    p.bias = d->bias;
    p.residual = d->residual;
    p.ldr = d->ldr;
    p.out = d->out;
    p.ldo = d->ldo;
    p.M = d->M;
    p.N = d->N;
    p.K = d->K;
    p.KB = d->K / 128;
    p.epi = d->epilogue;
    p.out_dtype = d->out_dtype;
    p.res_dtype = d->res_dtype;
    p.group_shift = 0;
    while ((1 << p.group_shift) < d->group) ++p.group_shift;
    p.flags = d->flags;
    p.eps = d->eps;
    p.inv_k = 1.0f / float(d->K);
    p.n_out = pl.tpu == 2 ? d->N / 2 : d->N;
    p.units = pl.units;
    p.uq = pl.units / pl.grid;
    p.ur = pl.units % pl.grid;
    p.nkw = pl.nkw;
    p.pitch = pl.pitch;
    p.upc = pl.upc;
    p.rbk = pl.rbk;
    p.wait_cycles = kWaitCycles;
    p.sm_w = pl.sm_w;
    p.sm_sc = pl.sm_sc;
    p.sm_bar = pl.sm_bar;
    p.sm_x = pl.sm_x;
    p.sm_xs = pl.sm_xs;
    p.sm_part = pl.sm_part;
    p.sm_misc = pl.sm_misc;
    p.sm_red = pl.sm_red;
    int rc = ensure_smem_attr(fn, pl.sm_total);
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kLeanThreads);
    cfg.dynamicSmemBytes = pl.sm_total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (d->flags & BQ_FLAG_PDL) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (pl.ks > 1) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = pl.ks;
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = na ? attr : nullptr;
    cfg.numAttrs = na;
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "GEMV launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // namespace bq
