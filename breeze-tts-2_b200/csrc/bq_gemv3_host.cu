// Host planning and launch of the v3 GEMV kernel (bq_gemv3.cuh).
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstring>
#include <map>
#include <mutex>

#include "bq_gemv3.cuh"
#include "bq_gemv3_kinst.h"
#include "bq_host.h"

namespace bq {

namespace {
constexpr uint32_t kTargetSmem = 110 * 1024;  // leaves room for a co-resident dependent CTA
constexpr int64_t kXBudget = 136 * 1024;       // staged activations per CTA
inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
int boxes(int fmt) { return fmt == BQ_W_BF16 ? 4 : (fmt == BQ_W_FP8_E4M3 || fmt == BQ_W_INT8) ? 2 : 1; }
bool int4fmt(int fmt) { return fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN; }
int gpk_of(const bq_gemv_desc* d) { return (d->wfmt == BQ_W_INT4_TINYGEMM && d->group < 128) ? 128 / d->group : 1; }
int tile_bytes(int fmt, int gpk) { return boxes(fmt) * kBoxBytes + (int4fmt(fmt) ? int(align_up(64 * gpk, 128)) : 0); }
}  // namespace

int gemv3_tile_bytes(int fmt, int gpk) { return tile_bytes(fmt, gpk); }
int gemv3_gpk(const bq_gemv_desc* d) { return gpk_of(d); }

int gemv3_rows_per_launch(const bq_gemv_desc* d) {
    const DeviceInfo* dev = device_info();
    const int optin = dev ? dev->smem_optin : 232448;
    // Without a norm the planner may split K across CTAs (up to 8 slices), so
    // only a slice of the activations is staged per CTA.
    const int KB = d->gamma ? d->K / kKB : (d->K / kKB + 7) / 8;
    const int nkbw = (KB + 7) / 8;
    const int64_t pitch = nkbw * 256 + 16;
    // smallest ring that still double-buffers: two slots of one two-tile unit per warp
    const int64_t ring = 8 * 2 * 2 * int64_t(tile_bytes(d->wfmt, gpk_of(d)));
    const int64_t xsum = int4fmt(d->wfmt) ? 8 * nkbw * gpk_of(d) * 2 * 64 : 0;  // int4 group sums
    const int64_t extra = 8 * nkbw * 256 + 4 * 8 * 2 * 2 * 512 + xsum;           // gamma, partials
    const int64_t budget = std::min<int64_t>(kXBudget, optin - ring - misc3_bytes(4, 16) - extra - 2048 - 8 * 256);
    const int r = int(budget / (8 * pitch));
    return std::max(1, std::min(16, r));
}

namespace {
// One plan for a K split into `ks` slices (ks = 1: every CTA covers all of K).
int plan_gemv3_ks(const bq_gemv_desc* d, int rows, Gemv3Plan* pl, int SMs, int ks) {
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    const int fmt = d->wfmt;
    const int KB = d->K / kKB;
    if (ks > KB) return BQ_ERR_SHAPE;
    Gemv3Plan P;
    std::memset(&P, 0, sizeof(P));
    P.rows = rows;
    P.mt = rows > 8 ? 2 : 1;
    P.ksplit = ks;
    P.nkbw = ((KB + ks - 1) / ks + 7) / 8;
    // k-block ranges exactly as the kernel derives them: slice [s*KB/ks, (s+1)*KB/ks), a warp
    // an eighth of it; all even lets the one-row kernels (two k-blocks per ring slot) drop
    // the half-slot path
    P.even_k = 1;
    for (int s = 0; s < ks; ++s) {
        const int n = (s + 1) * KB / ks - s * KB / ks;
        for (int w = 0; w < 8; ++w)
            if (((((w + 1) * n) >> 3) - ((w * n) >> 3)) & 1) P.even_k = 0;
    }
    P.xrow_pitch = P.nkbw * 256 + 16;
    P.gpk = gpk_of(d);
    const int SMu = std::max(1, SMs / ks);  // CTAs per K slice

    int64_t U;
    if (d->epilogue == BQ_EPI_SILU_MUL) {
        P.tpu = 2;
        U = (d->N / 2 + 15) / 16;
    } else {
        const int64_t u32 = (d->N + 31) / 32, u16 = (d->N + 15) / 16;
        auto rows_per_cta = [&](int64_t u, int r) {
            const int64_t g = std::min<int64_t>(SMu, u);
            return ((u + g - 1) / g) * r;
        };
        P.tpu = (ks > 1 || rows_per_cta(u16, 16) < rows_per_cta(u32, 32)) ? 1 : 2;  // rectangles: one-tile units
        U = P.tpu == 1 ? u16 : u32;
    }
    if (2 * U > kMaxUnits) return set_error(BQ_ERR_SHAPE, "N=%d too large for one launch", d->N);
    P.n_units = int(U);
    const int64_t T = U * KB;
    P.total_chunks = T;
    if ((T + 1) * int64_t(std::max(SMs, int((U + 3) / 4))) >= (int64_t(1) << 32))
        return set_error(BQ_ERR_SHAPE, "GEMV too large for one launch (N=%d, K=%d)", d->N, d->K);
    int upc_need;
    if (ks > 1) {
        // rectangles: a group of units x one K slice per CTA; the slices of a
        // unit are summed by the last CTA to finish it (split-mode epilogue)
        P.owned = 0;
        int64_t ngrp = std::min<int64_t>(SMu, U);
        if ((U + ngrp - 1) / ngrp > 4) ngrp = (U + 3) / 4;
        P.grid = int(ngrp * ks);
        upc_need = int((U + ngrp - 1) / ngrp);
        P.p_max = ks;
    } else if (U >= SMs / 2) {
        P.owned = 1;
        int64_t G = std::min<int64_t>(SMs, U);
        if ((U + G - 1) / G > 4) G = (U + 3) / 4;
        P.grid = int(G);
        upc_need = int((U + G - 1) / G);
    } else {
        P.owned = 0;
        const int64_t G = std::min<int64_t>(SMs, T);
        P.grid = int(G);
        const int64_t per = (T + G - 1) / G;
        upc_need = int(std::min<int64_t>(U, (per - 1 + KB - 1) / KB + 1));
        const int64_t cmin = T / G;
        P.p_max = int(std::min<int64_t>(G, (KB - 1 + cmin - 1) / cmin + 1));
    }
    if (upc_need > 4) return set_error(BQ_ERR_SHAPE, "internal: %d units per CTA", upc_need);
    P.upc = upc_need;
    const int ugm = 1;  // kernel ug_max()
    const int kps = P.mt == 1 ? 2 : 1;             // k-blocks per ring slot (kernel's KPS)
    const int nkp = (P.nkbw + kps - 1) / kps;      // ring slots per unit group and warp
    const uint32_t x_bytes = uint32_t(8 * (rows * P.xrow_pitch + 256));  // + one zero k-block per warp
    const uint32_t gamma_bytes = d->gamma ? uint32_t(8 * P.nkbw * 256) : 0u;
    const uint32_t xsum_bytes = int4fmt(fmt) ? uint32_t(8 * P.nkbw * P.gpk * P.mt * 64) : 0u;
    const int nq = rows >= 7 ? 4 : (rows + 1) / 2;  // lane groups holding real columns
    const uint32_t part_bytes = uint32_t(P.upc * 8 * P.tpu * P.mt * 128 * nq);
    auto layout = [&](int ug, int rs) {
        const uint32_t slot = uint32_t(kps * ug * P.tpu * tile_bytes(fmt, P.gpk));
        uint32_t o = 0;
        P.smem_ring = o;
        o += 8 * rs * slot;
        o = align_up(o, 16);
        P.smem_x = o;
        o += x_bytes;
        o = align_up(o, 16);
        P.smem_xsum = o;
        o += xsum_bytes;
        o = align_up(o, 16);
        P.smem_gamma = o;
        o += gamma_bytes;
        o = align_up(o, 16);
        P.smem_part = o;
        o += part_bytes;
        o = align_up(o, 16);
        P.smem_misc = o;
        o += misc3_bytes(P.upc, rows);
        return o;
    };
    // Largest unit group that still double-buffers within the co-residency
    // target; the deepest ring for it. Else one unit per slot, as deep as
    // the device allows.
    int ug = 0, rs = 0;
    for (int u = std::min(ugm, P.upc); u >= 1 && !ug; --u) {
        const int max_seq = std::min(kMaxRing, ((P.upc + u - 1) / u) * nkp);
        const int need = std::min(2, max_seq);
        if (layout(u, need) > kTargetSmem) continue;
        ug = u;
        rs = need;
        while (rs < max_seq && layout(u, rs + 1) <= kTargetSmem) ++rs;
    }
    if (!ug) {
        ug = 1;
        const int max_seq = std::min(kMaxRing, P.upc * nkp);
        rs = std::min(2, max_seq);
        while (rs > 1 && layout(1, rs) > uint32_t(dev->smem_optin)) --rs;
    }
    const uint32_t total = layout(ug, rs);
    if (total > uint32_t(dev->smem_optin))
        return set_error(BQ_ERR_SHAPE, "GEMV does not fit in shared memory (K=%d, rows=%d)", d->K, rows);
    P.ug = ug;
    P.slot_bytes = kps * ug * P.tpu * tile_bytes(fmt, P.gpk);
    P.ring_slots = rs;
    P.smem_total = total;
    P.ws_bytes = P.owned ? 0 : kCounterBytes + int64_t(U) * P.p_max * P.tpu * 2 * 128 * 4;
    *pl = P;
    return BQ_OK;
}
}  // namespace

namespace {
// The main loop's critical path under a plan: the most (unit, k-block) chunks
// one warp streams, in tiles, times the CTAs that share an SM. CTA ranges and
// warp k-ranges are derived as the kernel derives them; a warp whose eighth
// of K misses the CTA's range idles.
int64_t warp_load_max(const Gemv3Plan& P, int KB, int SMs) {
    const int ks = P.ksplit > 1 ? P.ksplit : 1;
    int64_t worst = 0;
    for (int cta = 0; cta < P.grid; ++cta) {
        int kb_lo = 0, kb_hi = KB;
        int64_t cb, ce;
        if (ks > 1) {
            const int ngrp = P.grid / ks, ugi = cta / ks, s = cta - ugi * ks;
            const int64_t u0 = int64_t(ugi) * P.n_units / ngrp, u1 = int64_t(ugi + 1) * P.n_units / ngrp;
            kb_lo = s * KB / ks;
            kb_hi = (s + 1) * KB / ks;
            cb = u0 * KB + kb_lo;
            ce = (u1 - 1) * KB + kb_hi;
        } else if (P.owned) {
            cb = int64_t(cta) * P.n_units / P.grid * KB;
            ce = int64_t(cta + 1) * P.n_units / P.grid * KB;
        } else {
            cb = int64_t(cta) * P.total_chunks / P.grid;
            ce = int64_t(cta + 1) * P.total_chunks / P.grid;
        }
        if (ce <= cb) continue;
        const int64_t uf = cb / KB, ul = (ce - 1) / KB;
        const int lo0 = int(cb - uf * KB), hi_last = int(ce - 1 - ul * KB);
        for (int w = 0; w < 8; ++w) {
            const int a = kb_lo + ((w * (kb_hi - kb_lo)) >> 3), b = kb_lo + (((w + 1) * (kb_hi - kb_lo)) >> 3);
            int64_t n = 0;
            for (int64_t u = uf; u <= ul; ++u) {
                const int lo = (ks > 1 || u == uf) ? std::max(a, lo0) : a;
                const int hi = (ks > 1 || u == ul) ? std::min(b - 1, hi_last) : b - 1;
                if (hi >= lo) n += hi - lo + 1;
            }
            worst = std::max(worst, n);
        }
    }
    return worst * P.tpu * ((P.grid + SMs - 1) / SMs);
}

// Plans depend only on the shape, format, epilogue, norm and device: cached,
// so a decode loop's repeated calls skip the layout search.
std::mutex g_plan_mu;
std::map<std::array<int, 9>, Gemv3Plan> g_plans;
int plan_gemv3_uncached(const bq_gemv_desc* d, int rows, Gemv3Plan* pl, int slots);
}  // namespace

int plan_gemv3(const bq_gemv_desc* d, int rows, Gemv3Plan* pl, int slots) {
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    const std::array<int, 9> key{dev->device, rows, d->N, d->K, d->wfmt, d->group, d->epilogue,
                                 d->gamma != nullptr ? 1 : 0, slots};
    {
        std::lock_guard<std::mutex> lk(g_plan_mu);
        auto it = g_plans.find(key);
        if (it != g_plans.end()) {
            *pl = it->second;
            return BQ_OK;
        }
    }
    const int rc = plan_gemv3_uncached(d, rows, pl, slots);
    if (rc == BQ_OK) {
        std::lock_guard<std::mutex> lk(g_plan_mu);
        if (g_plans.size() > 65536) g_plans.clear();
        g_plans.emplace(key, *pl);
    }
    return rc;
}

namespace {
int plan_gemv3_uncached(const bq_gemv_desc* d, int rows, Gemv3Plan* pl, int slots) {
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    // Without a norm (the row's sum of squares would need all of K), K may be
    // split across CTAs. Among the splits that leave room for a co-resident
    // dependent CTA, the one with the shortest per-warp critical path; a finer
    // split (more partial sums to reduce) must shorten it by a fifth.
    if (slots == 0 && !d->gamma && d->epilogue != BQ_EPI_SILU_MUL) {
        const int KB = d->K / kKB;
        // Long K (8 or more k-blocks per warp over the whole K: the down projections)
        // with int4 or bf16 weights and M <= 8: plan for two CTAs per SM, so that K
        // slices halve every warp's serial chain (depth down 1024x8192 M=2 7.46 ->
        // 6.63 us, backbone down 2048x8192 M=2 10.21 -> 8.76 us). Shorter K
        // (O 2048x2048: 3.86 -> 5.98 us) and fp8 / int8 measured slower that way.
        const bool two_per_sm = (int4fmt(d->wfmt) || d->wfmt == BQ_W_BF16) && rows <= 8 && KB / 8 >= 8;
        const int sms = two_per_sm ? 2 * dev->sm_count : dev->sm_count;
        bool found = false;
        int64_t best = 0;
        for (int ks = 1; ks <= 8; ks *= 2) {
            Gemv3Plan t;
            if (plan_gemv3_ks(d, rows, &t, sms, ks) != BQ_OK || t.smem_total > kTargetSmem) continue;
            if (two_per_sm && 2 * (int64_t(t.smem_total) + 1024) > int64_t(dev->smem_optin) + 1024) continue;
            const int64_t cost = warp_load_max(t, KB, sms);
            if (!found || 5 * cost <= 4 * best) {
                *pl = t;
                best = cost;
                found = true;
            }
        }
        if (found) return BQ_OK;
        // nothing leaves room for a dependent CTA: the finest split that fits at all
        for (int ks = 8; ks >= 2; ks /= 2)
            if (plan_gemv3_ks(d, rows, pl, dev->sm_count, ks) == BQ_OK) return BQ_OK;
    }
    if (slots == 0) {
        // Two CTAs of this GEMV per SM when both fit one SM's shared memory (the
        // SM's capacity is the per-block opt-in plus 1 KB, each block reserving
        // 1 KB): every CTA's serial chain (staging, group sums, main loop,
        // epilogue) covers half as many units, which outweighs parking the next
        // launch beside it. Plans that would need two waves keep one CTA per SM,
        // and so do the f16-activation formats (fp8, int8) and M > 8, where it
        // measured no better.
        Gemv3Plan t2;
        if ((int4fmt(d->wfmt) || d->wfmt == BQ_W_BF16) && rows <= 8 &&
            plan_gemv3_ks(d, rows, &t2, 2 * dev->sm_count, 1) == BQ_OK &&
            2 * (int64_t(t2.smem_total) + 1024) <= int64_t(dev->smem_optin) + 1024) {
            *pl = t2;
            return BQ_OK;
        }
    }
    return plan_gemv3_ks(d, rows, pl, slots > 0 ? slots : dev->sm_count, 1);
}
}  // namespace

void fill_gemv3_params(const bq_gemv_desc* d, const Gemv3Plan& pl, int row0, void* workspace, Gemv3Params* out) {
    Gemv3Params& p = *out;
    std::memset(&p, 0, sizeof(p));
    p.M = pl.rows;
    p.N = d->N;
    p.K = d->K;
    p.KB = d->K / kKB;
    p.epi = d->epilogue;
    p.group = d->group;
    p.x_dtype = d->x_dtype;
    p.out_dtype = d->out_dtype;
    p.res_dtype = d->res_dtype;
    p.flags = d->flags;
    p.eps = d->eps;
    p.n_half = d->N / 2;
    p.tpu = pl.tpu;
    p.n_units = pl.n_units;
    p.owned = pl.owned;
    p.grid = pl.grid;
    p.total_chunks = pl.total_chunks;
    p.ug = pl.ug;
    p.ring_slots = pl.ring_slots;
    p.slot_bytes = pl.slot_bytes;
    p.nkbw = pl.nkbw;
    p.p_max = pl.p_max;
    p.xrow_pitch = pl.xrow_pitch;
    p.upc = pl.upc;
    p.ksplit = pl.ksplit > 1 ? pl.ksplit : 1;
    p.smem_ring = pl.smem_ring;
    p.smem_x = pl.smem_x;
    p.smem_xsum = pl.smem_xsum;
    p.smem_gamma = pl.smem_gamma;
    p.smem_part = pl.smem_part;
    p.smem_misc = pl.smem_misc;
    p.group_shift = 0;
    while ((1 << p.group_shift) < d->group) ++p.group_shift;
    const int xs = dtype_size(d->x_dtype), os = dtype_size(d->out_dtype), rsz = dtype_size(d->res_dtype);
    p.x = static_cast<const char*>(d->x) + int64_t(row0) * d->ldx * xs;
    p.x_bulk = (d->x_dtype == BQ_DT_BF16 && (reinterpret_cast<uintptr_t>(p.x) & 15) == 0 && (d->ldx % 8) == 0) ? 1 : 0;
    p.ldx = d->ldx;
    p.w = d->w;
    p.gamma = d->gamma;
    p.scale = d->scale;
    p.bias = d->bias;
    p.residual = d->residual ? static_cast<const char*>(d->residual) + int64_t(row0) * d->ldr * rsz : nullptr;
    p.ldr = d->ldr;
    p.res_bulk = (p.residual && (d->res_dtype == BQ_DT_BF16 || d->res_dtype == BQ_DT_F16 || d->res_dtype == BQ_DT_F32) &&
                  (reinterpret_cast<uintptr_t>(p.residual) & 15) == 0 && (d->ldr * rsz) % 16 == 0)
                     ? 1
                     : 0;
    p.out = static_cast<char*>(d->out) + int64_t(row0) * d->ldo * os;
    p.ldo = d->ldo;
    if (!pl.owned) {
        p.counters = static_cast<unsigned int*>(workspace);
        p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kCounterBytes);
    }
}

int launch_gemv3(const bq_gemv_desc* d, const Gemv3Plan& pl, int row0, void* workspace, cudaStream_t stream) {
    const int fmt = d->wfmt;
    const void* fn = nullptr;
    if (int4fmt(fmt))
        fn = gemv3_kernel_int4(fmt, pl.mt, pl.tpu, pl.gpk, pl.ksplit > 1, pl.even_k != 0);
    else if (fmt == BQ_W_BF16)
        fn = gemv3_kernel_bf16(pl.mt, pl.tpu, pl.ksplit > 1, pl.even_k != 0);
    else
        fn = gemv3_kernel_f8(fmt, pl.mt, pl.tpu, pl.ksplit > 1, pl.even_k != 0);
    if (!fn) return set_error(BQ_ERR_FORMAT, "no GEMV kernel for format %d (group %d)", fmt, d->group);

    Gemv3Params p;
    fill_gemv3_params(d, pl, row0, workspace, &p);
    int rc = ensure_smem_attr(fn, pl.smem_total);
    if (rc) return rc;

    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads3);
    cfg.dynamicSmemBytes = pl.smem_total;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (d->flags & BQ_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "GEMV launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // namespace bq
