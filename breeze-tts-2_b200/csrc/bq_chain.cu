// Host side of the decode chain: one cooperative launch running a list of
// GEMVs (bq_gemv_chain_*). The op table, the grid-barrier words and the
// split-K scratch live in the caller's workspace:
//   [0, 256)                  barrier {count, generation}
//   [256, 256 + n * op size)  op table (Gemv3Params, written by prepare)
//   then, 256-aligned          split-K counters and partial sums
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "bq_gemv3.cuh"
#include "bq_gemv3_kinst.h"
#include "bq_host.h"

namespace bq {

int validate_gemv(const bq_gemv_desc* d);

namespace {
constexpr int64_t kBarrierBytes = 256;
inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }

struct ChainPlan {
    int n, mt, gpk, fmt, grid;
    uint32_t smem;
    int64_t table_off, split_off, ws_bytes;
    std::vector<Gemv3Plan> ops;
};

const void* chain_kernel(int fmt, int mt, int gpk) {
    if (fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN) return gemv_chain_kernel_int4(fmt, mt, gpk);
    if (fmt == BQ_W_BF16) return gemv_chain_kernel_bf16(mt);
    return gemv_chain_kernel_f8(fmt, mt);
}

int plan_chain(const bq_gemv_desc* descs, int n, ChainPlan* cp) {
    if (!descs || n < 1) return set_error(BQ_ERR_INVALID_ARG, "chain needs at least one GEMV");
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    cp->n = n;
    cp->fmt = descs[0].wfmt;
    cp->gpk = gemv3_gpk(&descs[0]);
    const int M = descs[0].M;
    cp->mt = M > 8 ? 2 : 1;
    for (int i = 0; i < n; ++i) {
        const bq_gemv_desc* d = &descs[i];
        int rc = validate_gemv(d);
        if (rc) {
            char msg[256];
            std::strncpy(msg, bq_last_error_string(), sizeof(msg) - 1);
            msg[sizeof(msg) - 1] = 0;
            return set_error(rc, "chain op %d: %s", i, msg);
        }
        if (d->gamma && (reinterpret_cast<uintptr_t>(d->gamma) & 15))
            return set_error(BQ_ERR_ALIGN, "chain op %d: gamma must be 16-byte aligned", i);
        if (d->wfmt != cp->fmt || gemv3_gpk(d) != cp->gpk || d->M != M)
            return set_error(BQ_ERR_SHAPE, "chain op %d: every GEMV of a chain needs the same format, group and M", i);
    }
    // Two CTAs per SM when the shared layout allows a double-buffered ring,
    // else one; a single-buffered ring only as the last resort.
    const int tb = gemv3_tile_bytes(cp->fmt, cp->gpk);
    // BQ_CHAIN_CTAS_PER_SM=1 pins one CTA per SM (for comparisons)
    const char* env = std::getenv("BQ_CHAIN_CTAS_PER_SM");
    const int first = (env && std::atoi(env) == 1) ? 1 : 0;
    for (int attempt = first; attempt < 3; ++attempt) {
        const int per_sm = attempt == 0 ? 2 : 1;
        const int min_rs = attempt < 2 ? 2 : 1;
        const int slots = per_sm * dev->sm_count;
        // per-CTA dynamic shared memory: 228 KB per SM, 1 KB reserved per CTA,
        // 1 KB kept for the kernel's static op slots
        const uint32_t budget =
            std::min<uint32_t>(uint32_t(dev->smem_optin) - 1024u, (233472u - 1024u * per_sm) / per_sm - 1024u);
        cp->grid = slots;
        cp->ops.assign(n, Gemv3Plan());
        uint32_t x_max = 0, g_max = 0, part_max = 0, xs_max = 0;
        int64_t split_need = 0;
        bool ok = true;
        for (int i = 0; i < n && ok; ++i) {
            const bq_gemv_desc* d = &descs[i];
            if (plan_gemv3(d, M, &cp->ops[i], slots) != BQ_OK) {
                ok = false;
                break;
            }
            const Gemv3Plan& pl = cp->ops[i];
            x_max = std::max<uint32_t>(x_max, uint32_t(8 * (M * pl.xrow_pitch + 256)));
            if (d->gamma) g_max = std::max<uint32_t>(g_max, uint32_t(8 * pl.nkbw * 256));
            if (cp->fmt == BQ_W_INT4_TINYGEMM || cp->fmt == BQ_W_INT4_PLAIN)
                xs_max = std::max<uint32_t>(xs_max, uint32_t(8 * pl.nkbw * pl.gpk * pl.mt * 64));
            const int nq = M >= 7 ? 4 : (M + 1) / 2;
            part_max = std::max<uint32_t>(part_max, uint32_t(pl.upc * 8 * pl.tpu * pl.mt * 128 * nq));
            split_need = std::max(split_need, pl.ws_bytes);
        }
        if (!ok) continue;
        // shared layout for every op: ring | x | gamma | partials | misc
        int upc_max = 1;
        for (int i = 0; i < n; ++i) upc_max = std::max(upc_max, cp->ops[i].upc);
        const uint32_t misc = misc3_bytes(upc_max, M);
        const uint32_t fixed = align_up(x_max, 16) + align_up(xs_max, 16) + align_up(g_max, 16) + align_up(part_max, 16) + misc;
        if (fixed >= budget) continue;
        const uint32_t ring_w = ((budget - fixed) / 8) / 128 * 128;  // ring bytes per warp
        const uint32_t smem_x = 8 * ring_w;
        const uint32_t smem_xsum = align_up(smem_x + x_max, 16);
        const uint32_t smem_gamma = align_up(smem_xsum + xs_max, 16);
        const uint32_t smem_part = align_up(smem_gamma + g_max, 16);
        const uint32_t smem_misc = align_up(smem_part + part_max, 16);
        for (int i = 0; i < n && ok; ++i) {
            Gemv3Plan& pl = cp->ops[i];
            const int ugm = 1;  // kernel ug_max()
            const int kps = pl.mt == 1 ? 2 : 1;
            const int nkp = (pl.nkbw + kps - 1) / kps;
            int ug = std::min(ugm, pl.upc), rs = 0;
            for (; ug >= 1; --ug) {
                const int slot = kps * ug * pl.tpu * tb;
                const int max_seq = std::min(kMaxRing, ((pl.upc + ug - 1) / ug) * nkp);
                rs = std::min<int>(max_seq, int(ring_w / uint32_t(slot)));
                if (rs >= std::min(min_rs, max_seq)) break;
            }
            if (ug < 1 || rs < 1) {
                ok = false;
                break;
            }
            pl.ug = ug;
            pl.slot_bytes = kps * ug * pl.tpu * tb;
            pl.ring_slots = rs;
            pl.smem_ring = 0;
            pl.smem_x = smem_x;
            pl.smem_xsum = smem_xsum;
            pl.smem_gamma = smem_gamma;
            pl.smem_part = smem_part;
            pl.smem_misc = smem_misc;
        }
        if (!ok) continue;
        cp->smem = smem_misc + misc;
        for (int i = 0; i < n; ++i) cp->ops[i].smem_total = cp->smem;
        cp->table_off = kBarrierBytes;
        cp->split_off = align256(kBarrierBytes + int64_t(n) * int64_t(sizeof(Gemv3Params)));
        cp->ws_bytes = cp->split_off + split_need;
        return BQ_OK;
    }
    return set_error(BQ_ERR_SHAPE, "chain of %d GEMVs with M=%d does not fit in shared memory", n, M);
}
}  // namespace

}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_gemv_chain_workspace_bytes(const bq_gemv_desc* descs, int32_t n, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    ChainPlan cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    *bytes = size_t(cp.ws_bytes);
    return BQ_OK;
}

int32_t bq_gemv_chain_prepare(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes) {
    ChainPlan cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    if (!workspace || int64_t(workspace_bytes) < cp.ws_bytes)
        return set_error(BQ_ERR_WORKSPACE, "chain workspace of %zu bytes given, %lld needed", workspace_bytes,
                         (long long)cp.ws_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
    char* ws = static_cast<char*>(workspace);
    std::vector<Gemv3Params> table(n);
    for (int i = 0; i < n; ++i) fill_gemv3_params(&descs[i], cp.ops[i], 0, ws + cp.split_off, &table[i]);
    cudaError_t e = cudaMemset(ws, 0, size_t(cp.table_off));
    if (e == cudaSuccess) e = cudaMemset(ws + cp.split_off, 0, size_t(cp.ws_bytes - cp.split_off));
    if (e == cudaSuccess) e = cudaMemcpy(ws + cp.table_off, table.data(), sizeof(Gemv3Params) * size_t(n), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "chain prepare: %s", cudaGetErrorString(e));
    return BQ_OK;
}

int32_t bq_gemv_chain_launch(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes,
                             void* stream) {
    ChainPlan cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    if (!workspace || int64_t(workspace_bytes) < cp.ws_bytes)
        return set_error(BQ_ERR_WORKSPACE, "chain workspace of %zu bytes given, %lld needed", workspace_bytes,
                         (long long)cp.ws_bytes);
    const void* fn = chain_kernel(cp.fmt, cp.mt, cp.gpk);
    if (!fn) return set_error(BQ_ERR_FORMAT, "no chain kernel for format %d", cp.fmt);
    rc = ensure_smem_attr(fn, cp.smem);
    if (rc) return rc;
    int per_sm = 0;
    const DeviceInfo* dev = device_info();
    const int want = cp.grid / dev->sm_count;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kThreads3, cp.smem);
    if (e != cudaSuccess || per_sm < want)
        return set_error(BQ_ERR_CUDA, "chain kernel cannot keep %d CTAs per SM (%d, %s)", want, per_sm, cudaGetErrorString(e));
    char* ws = static_cast<char*>(workspace);
    const Gemv3Params* ops = reinterpret_cast<const Gemv3Params*>(ws + cp.table_off);
    int n_ops = n;
    unsigned int* bar = reinterpret_cast<unsigned int*>(ws);
    void* args[] = {&ops, &n_ops, &bar};
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(cp.grid);
    cfg.blockDim = dim3(kThreads3);
    cfg.dynamicSmemBytes = cp.smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    int na = 1;
    if (descs[0].flags & BQ_FLAG_PDL) {
        attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[1].val.programmaticStreamSerializationAllowed = 1;
        na = 2;
    }
    cfg.attrs = attr;
    cfg.numAttrs = na;
    e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "chain launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
