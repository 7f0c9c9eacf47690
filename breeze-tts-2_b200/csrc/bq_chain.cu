// Host side of the decode chain (bq_gemv_chain_*): planning, the op table and
// the launch of the persistent kernel in bq_chain.cuh.
//
// Workspace layout (caller-provided, 256-byte aligned, sized by
// bq_gemv_chain_workspace_bytes):
//   [0, 256)                   ChainHeader: epoch, wait limit, start flag, finish count
//   [256, 256 + 128 n)         per-op completion counters, one 128-byte line each
//   then (256-aligned)         op table: n ChainOp
//   then (256-aligned, each)   tile-major copies of the int4 ops' scale/zero pairs,
//                              [N/16][K/g][16][2] bf16, written by prepare
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <vector>

#include "bq_chain.cuh"
#include "bq_host.h"

namespace bq {

int validate_gemv(const bq_gemv_desc* d);

namespace {
inline int64_t align256(int64_t v) { return (v + 255) / 256 * 256; }
inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
bool is_int4(int fmt) { return fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN; }
int row_kb_bytes(int fmt) { return fmt == BQ_W_BF16 ? 256 : (fmt == BQ_W_FP8_E4M3 || fmt == BQ_W_INT8) ? 128 : 64; }

struct ChainPlanH {
    int n = 0, M = 0, mt = 1, grid = 0, R = 0;
    uint32_t slot = 0, smem = 0, smem_x = 0, smem_xsum = 0, smem_part = 0, smem_misc = 0, smem_bar = 0;
    uint32_t xw_bytes = 0, xw_pitch = 0, xsum_w_bytes = 0, part_bytes = 0;
    int64_t off_counters = 256, off_table = 0, ws_bytes = 0;
    std::vector<ChainOp> ops;
    std::vector<int64_t> scale_off;  // workspace offset of each int4 op's tile-major scales (-1: none)
};

// Scale bytes of one 16-row piece for a chunk of kbc k-blocks.
uint32_t piece_scale_bytes(const bq_gemv_desc* d, int kbc) {
    if (is_int4(d->wfmt)) return uint32_t(kbc * kKB / d->group) * 64u;
    if (d->wfmt == BQ_W_FP8_E4M3 || d->wfmt == BQ_W_INT8) return 64u;
    return 0u;
}

int plan_chain(const bq_gemv_desc* descs, int n, ChainPlanH* cp) {
    if (!descs || n < 1) return set_error(BQ_ERR_INVALID_ARG, "chain needs at least one GEMV");
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    cp->n = n;
    cp->M = descs[0].M;
    cp->mt = cp->M > 8 ? 2 : 1;
    cp->grid = dev->sm_count;
    if (cp->M > 16) return set_error(BQ_ERR_SHAPE, "the decode chain takes at most 16 rows (got %d)", cp->M);
    auto fail = [&](int i, int code, const char* what) {
        return set_error(code, "chain op %d: %s", i, what);
    };
    for (int i = 0; i < n; ++i) {
        const bq_gemv_desc* d = &descs[i];
        int rc = validate_gemv(d);
        if (rc) {
            char msg[256];
            std::strncpy(msg, bq_last_error_string(), sizeof(msg) - 1);
            msg[sizeof(msg) - 1] = 0;
            return set_error(rc, "chain op %d: %s", i, msg);
        }
        if (d->M != cp->M) return fail(i, BQ_ERR_SHAPE, "every GEMV of a chain has the same M");
        const int n_tile_rows = d->epilogue == BQ_EPI_SILU_MUL ? d->N / 2 : d->N;
        if (n_tile_rows % 16) return fail(i, BQ_ERR_SHAPE, "N (N / 2 with SiLU*up) must be a multiple of 16");
        if (d->x_dtype != BQ_DT_BF16 || (reinterpret_cast<uintptr_t>(d->x) & 15) || (d->ldx % 8))
            return fail(i, BQ_ERR_ALIGN, "x must be bf16 with 16-byte aligned rows");
        if (d->gamma && (reinterpret_cast<uintptr_t>(d->gamma) & 15)) return fail(i, BQ_ERR_ALIGN, "gamma must be 16-byte aligned");
        if (d->epilogue == BQ_EPI_ADD_RESIDUAL &&
            (d->res_dtype != BQ_DT_BF16 || (reinterpret_cast<uintptr_t>(d->residual) & 15) || (d->ldr % 8)))
            return fail(i, BQ_ERR_ALIGN, "the residual must be bf16 with 16-byte aligned rows");
        if ((d->wfmt == BQ_W_FP8_E4M3 || d->wfmt == BQ_W_INT8) && (reinterpret_cast<uintptr_t>(d->scale) & 15))
            return fail(i, BQ_ERR_ALIGN, "the row scales must be 16-byte aligned");
        const int tiles = n_tile_rows / 16;
        if ((tiles + cp->grid - 1) / cp->grid > kChainMaxTiles)
            return fail(i, BQ_ERR_SHAPE, "too many output rows for one chain op");
    }
    // chunking and shared-memory layout for a chunk-size cap; more ring slots win
    for (const uint32_t cap : {34u * 1024u, 17u * 1024u}) {
        ChainPlanH P = *cp;
        P.ops.assign(n, ChainOp());
        uint32_t slot = 0;
        int nkw_max = 0, gpk_max = 1;
        bool ok = true;
        for (int i = 0; i < n && ok; ++i) {
            const bq_gemv_desc* d = &descs[i];
            const int KB = d->K / kKB, rkb = row_kb_bytes(d->wfmt);
            const int pieces = d->epilogue == BQ_EPI_SILU_MUL ? 2 : 1;
            int kbc = 0;
            for (int nch = 1; nch <= KB; ++nch) {
                if (KB % nch) continue;
                const int c = KB / nch;
                if (is_int4(d->wfmt) && (c * kKB) % d->group) continue;  // whole groups per chunk
                const uint32_t bytes = uint32_t(pieces) * (uint32_t(c) * 16u * uint32_t(rkb) + piece_scale_bytes(d, c));
                if (bytes <= cap) {
                    kbc = c;
                    break;
                }
            }
            if (!kbc) {
                ok = false;
                break;
            }
            ChainOp& o = P.ops[i];
            std::memset(&o, 0, sizeof(o));
            o.fmt = d->wfmt;
            o.M = d->M;
            o.N = d->N;
            o.K = d->K;
            o.KB = KB;
            o.group = d->group;
            o.gpk = (d->wfmt == BQ_W_INT4_TINYGEMM && d->group < 128) ? 128 / d->group : 1;
            o.epi = d->epilogue;
            o.norm = d->gamma ? 1 : 0;
            o.x_dtype = d->x_dtype;
            o.out_dtype = d->out_dtype;
            o.res_dtype = d->res_dtype;
            o.flags = d->flags;
            o.eps = d->eps;
            o.n_half = d->N / 2;
            o.pieces = pieces;
            o.tiles = (pieces == 2 ? d->N / 2 : d->N) / 16;
            o.kbc = kbc;
            o.nchunk = KB / kbc;
            o.wpiece = uint32_t(kbc) * 16u * uint32_t(rkb);
            o.piece_bytes = o.wpiece + piece_scale_bytes(d, kbc);
            o.chunk_bytes = uint32_t(pieces) * o.piece_bytes;
            o.row_copies = d->wfmt == BQ_W_INT4_TINYGEMM ? 2 : (o.nchunk == 1 ? 1 : 16);
            o.x = d->x;
            o.ldx = d->ldx;
            o.w = d->w;
            o.scale = d->scale;
            o.gamma = d->gamma;
            o.bias = d->bias;
            o.residual = d->residual;
            o.ldr = d->ldr;
            o.out = d->out;
            o.ldo = d->ldo;
            slot = std::max(slot, o.chunk_bytes);
            if (o.norm) slot = std::max(slot, uint32_t(d->K) * 2u);
            nkw_max = std::max(nkw_max, o.nchunk * ((kbc + 7) / 8));
            gpk_max = std::max(gpk_max, o.gpk);
        }
        if (!ok) continue;
        slot = align_up(slot, 128);
        // tile rotation: op i's tiles start where op i-1's ended, spreading every CTA's weight bytes evenly
        int64_t base = 0;
        for (int i = 0; i < n; ++i) {
            P.ops[i].base = int(base % P.grid);
            base += P.ops[i].tiles;
        }
        const int M = P.M, MT = P.mt;
        P.xw_pitch = uint32_t(nkw_max) * 256u + 16u;
        P.xw_bytes = align_up(uint32_t(M) * P.xw_pitch + 256u, 16);
        bool any_int4 = false;
        for (int i = 0; i < n; ++i) any_int4 |= is_int4(descs[i].wfmt);
        P.xsum_w_bytes = any_int4 ? uint32_t(nkw_max * gpk_max) * 16u * 4u : 0u;  // [block][sub-group][16 rows] fp32
        const int nq = M >= 7 ? 4 : (M + 1) / 2;
        P.part_bytes = uint32_t(8 * 2 * MT * 8 * nq) * 16u;  // one tile's partial sums
        const uint32_t fixed = 8 * P.xw_bytes + 8 * P.xsum_w_bytes + kChainMaxTiles * P.part_bytes + chain_misc_bytes();
        // the kernel's static shared memory (abort flag, epoch) and 1 KB per-CTA reserve fit in the opt-in limit
        const uint32_t budget = uint32_t(dev->smem_optin) - 256u;
        if (fixed + 2 * (slot + 16) > budget) continue;
        P.R = int(std::min<uint32_t>((budget - fixed) / (slot + 16), 64u));
        P.slot = slot;
        uint32_t o = 0;
        o += uint32_t(P.R) * slot;
        P.smem_x = o;
        o += 8 * P.xw_bytes;
        P.smem_xsum = o;
        o += 8 * P.xsum_w_bytes;
        P.smem_part = o;
        o += kChainMaxTiles * P.part_bytes;
        P.smem_misc = o;
        o += chain_misc_bytes();
        o = align_up(o, 16);
        P.smem_bar = o;
        o += 16u * uint32_t(P.R);
        P.smem = o;
        if (P.R < 3 && cap != 17u * 1024u) {
            *cp = P;  // keep as a fallback, try smaller chunks
            continue;
        }
        *cp = P;
        break;
    }
    if (cp->R < 2) return set_error(BQ_ERR_SHAPE, "a chain of %d GEMVs with M=%d does not fit in shared memory", n, cp->M);
    // workspace: header, counters, op table, int4 scale copies
    cp->off_counters = 256;
    cp->off_table = align256(cp->off_counters + int64_t(n) * kCounterStride * 4);
    int64_t off = align256(cp->off_table + int64_t(n) * int64_t(sizeof(ChainOp)));
    cp->scale_off.assign(n, -1);
    for (int i = 0; i < n; ++i) {
        const bq_gemv_desc* d = &descs[i];
        if (!is_int4(d->wfmt)) continue;
        cp->scale_off[i] = off;
        off = align256(off + int64_t(d->N) * (d->K / d->group) * 4);
    }
    cp->ws_bytes = off;
    return BQ_OK;
}

// scales_zeros [K/g, N, 2] bf16 -> tile-major [N/16][K/g][16][2]: one 32-bit pair per thread.
__global__ void scales_tile_major_kernel(const uint32_t* __restrict__ src, uint32_t* __restrict__ dst, int n, int groups) {
    const int64_t total = int64_t(n) * groups;
    for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
        const int64_t g = i / n, row = i - g * n;  // source order: coalesced reads
        dst[((row / 16) * groups + g) * 16 + (row & 15)] = src[i];
    }
}

template <int MT>
const void* chain_kernel_mt(int fmt, int gpk) {
    switch (fmt) {
        case BQ_W_INT4_TINYGEMM:
            if (gpk == 4) return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_INT4_TINYGEMM, 4>);
            if (gpk == 2) return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_INT4_TINYGEMM, 2>);
            return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_INT4_TINYGEMM, 1>);
        case BQ_W_INT4_PLAIN: return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_INT4_PLAIN, 1>);
        case BQ_W_FP8_E4M3: return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_FP8_E4M3, 1>);
        case BQ_W_INT8: return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_INT8, 1>);
        case BQ_W_BF16: return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, BQ_W_BF16, 1>);
        default: return reinterpret_cast<const void*>(&gemv_chain_kernel<MT, -1, 1>);  // mixed formats
    }
}

// The kernel for a chain: specialised to its format when every op shares one.
const void* chain_kernel(const ChainPlanH& cp) {
    int fmt = cp.ops[0].fmt, gpk = cp.ops[0].gpk;
    for (const ChainOp& o : cp.ops)
        if (o.fmt != fmt || o.gpk != gpk) fmt = -1;
    return cp.mt == 1 ? chain_kernel_mt<1>(fmt, gpk) : chain_kernel_mt<2>(fmt, gpk);
}
}  // namespace

}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_gemv_chain_workspace_bytes(const bq_gemv_desc* descs, int32_t n, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    ChainPlanH cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    *bytes = size_t(cp.ws_bytes);
    return BQ_OK;
}

int32_t bq_gemv_chain_prepare_ex(const bq_gemv_desc* descs, int32_t n, const bq_chain_options* opts, void* workspace,
                                 size_t workspace_bytes) {
    ChainPlanH cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    if (!workspace || int64_t(workspace_bytes) < cp.ws_bytes)
        return set_error(BQ_ERR_WORKSPACE, "chain workspace of %zu bytes given, %lld needed", workspace_bytes,
                         (long long)cp.ws_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
    char* ws = static_cast<char*>(workspace);
    ChainHeader h;
    std::memset(&h, 0, sizeof(h));
    if (opts) {
        h.wait_cycles = (long long)opts->wait_cycles;
        h.start_flag = opts->start_flag;
        h.start_target = opts->start_target;
    }
    std::vector<ChainOp> table = cp.ops;
    cudaError_t e = cudaSuccess;
    for (int i = 0; i < n && e == cudaSuccess; ++i) {
        if (cp.scale_off[i] < 0) continue;
        const bq_gemv_desc* d = &descs[i];
        uint32_t* dst = reinterpret_cast<uint32_t*>(ws + cp.scale_off[i]);
        const int groups = d->K / d->group;
        const int64_t total = int64_t(d->N) * groups;
        const int blocks = int(std::min<int64_t>((total + 255) / 256, 4096));
        scales_tile_major_kernel<<<blocks, 256>>>(static_cast<const uint32_t*>(d->scale), dst, d->N, groups);
        e = cudaGetLastError();
        table[i].scale = dst;
    }
    if (e == cudaSuccess) e = cudaMemcpy(ws, &h, sizeof(h), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(ws + cp.off_counters, 0, size_t(cp.off_table - cp.off_counters));
    if (e == cudaSuccess)
        e = cudaMemcpy(ws + cp.off_table, table.data(), sizeof(ChainOp) * size_t(n), cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "chain prepare: %s", cudaGetErrorString(e));
    return BQ_OK;
}

int32_t bq_gemv_chain_prepare(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes) {
    return bq_gemv_chain_prepare_ex(descs, n, nullptr, workspace, workspace_bytes);
}

int32_t bq_gemv_chain_launch(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes,
                             void* stream) {
    ChainPlanH cp;
    int rc = plan_chain(descs, n, &cp);
    if (rc) return rc;
    if (!workspace || int64_t(workspace_bytes) < cp.ws_bytes)
        return set_error(BQ_ERR_WORKSPACE, "chain workspace of %zu bytes given, %lld needed", workspace_bytes,
                         (long long)cp.ws_bytes);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
    const void* fn = chain_kernel(cp);
    rc = ensure_smem_attr(fn, cp.smem);
    if (rc) return rc;
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, kChainThreads, cp.smem);
    if (e != cudaSuccess || per_sm < 1)
        return set_error(BQ_ERR_CUDA, "chain kernel does not fit one CTA per SM (%u bytes of shared memory): %s",
                         cp.smem, cudaGetErrorString(e));
    char* ws = static_cast<char*>(workspace);
    ChainArgs a;
    std::memset(&a, 0, sizeof(a));
    a.ops = reinterpret_cast<const ChainOp*>(ws + cp.off_table);
    a.n_ops = n;
    a.ring_slots = cp.R;
    a.slot_bytes = cp.slot;
    a.smem_x = cp.smem_x;
    a.smem_xsum = cp.smem_xsum;
    a.smem_part = cp.smem_part;
    a.smem_misc = cp.smem_misc;
    a.smem_bar = cp.smem_bar;
    a.xw_bytes = cp.xw_bytes;
    a.xw_pitch = cp.xw_pitch;
    a.xsum_w_bytes = cp.xsum_w_bytes;
    a.part_bytes = cp.part_bytes;
    a.counters = reinterpret_cast<unsigned int*>(ws + cp.off_counters);
    a.hdr = reinterpret_cast<ChainHeader*>(ws);
    void* args[] = {&a};
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(cp.grid);
    cfg.blockDim = dim3(kChainThreads);
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
