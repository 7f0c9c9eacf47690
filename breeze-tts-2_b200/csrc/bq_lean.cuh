// Resident-slice GEMV for one or two activation rows (the decode step and
// BASELINE config 1): out = epilogue(norm(x) @ W^T), one launch, no global
// scratch.
//
// Why a second small-M kernel: a decode GEMV is a chain of dependent launches,
// and its time per call is the length of the serial path after the
// programmatic-dependent-launch (PDL) wait, not the weight bytes. This kernel
// moves everything that does not depend on the previous kernel in front of
// that wait, and keeps what follows it short:
//
//  * One CTA per SM (148), 8 warps, at most ~110 KB of shared memory where the
//    shape allows, so the next launch's CTA parks beside the running one. A CTA
//    owns whole 16-row units (SiLU*up: 16 gate + 16 up rows): no partial sums
//    in global memory, no counters. Shapes with fewer units than half the SMs
//    split K in two across a cluster of two CTAs per unit instead, the partial
//    sums meeting in distributed shared memory (KS below).
//  * Before the wait: the CTA's entire weight slice goes to shared memory as
//    one bulk copy (TMA engine) per half -- a CTA's rows are contiguous in
//    every layout -- completing on an mbarrier; the int4 scale/zero rows of
//    each warp's k-blocks as 16-byte cp.async copies; gamma, per-row scales and
//    bias to registers. The bulk copy keeps the load/store path free, so the
//    activation load after the wait does not queue behind ~50 KB of weight
//    copies (its own, and those of the next launch parked beside it).
//  * After the wait: each warp loads its K range of x straight into registers
//    (one 16-byte load per lane and chunk), multiplies by gamma, accumulates
//    sum(x^2), rounds to bf16 (int4 / bf16 weights) or to f16 scaled by a
//    power of two (fp8 / int8), sums each int4 group with shuffles, and stores
//    the staged rows for the B fragments. No block barrier before the main
//    loop: a warp only reads its own K range.
//  * Main loop, k-block-major: the activation fragments of a k-block are loaded
//    once and used for every unit of the CTA (independent accumulators, so the
//    MMA latency of one unit hides behind the others; one-tile shapes run the
//    unit loop straight-line over the plan's exact unit count).
//  * int4: codes become bf16 128 + q with one LOP3 per pair (exact); the group's
//    scale and zero are applied in fp32 per group: s (C - (128 + o) X) + z X
//    with X the staged activations' group sum (o = 8 tinygemm, 0 plain).
//  * Epilogue: one block barrier, then each thread finishes output elements:
//    eight warp partials summed in warp order (deterministic), 1/rms, per-row
//    scale, bias, SiLU*up or + residual (prefetched before the barrier), store.
//
// Same contract and numerics as bq_gemv (models/fused/kernels.py:334-351,
// models/int4_linear.py:99-109, models/fp8_linear.py:68-83,
// models/int8_linear.py:50-53).
#pragma once

#include <cuda_runtime.h>

#include "bq_device.cuh"
#include "bq_gemv3.cuh"
#include "bq_host.h"

namespace bq {

constexpr int kLeanThreads = 256;
constexpr int kLeanMaxChunks = 8;  // 16-byte x chunks per lane (M * ceil(KB / 8) <= 16)

struct LeanParams {
    const __nv_bfloat16* x;
    int64_t ldx;
    const __nv_bfloat16* gamma;
    const void* w;
    const void* scale;
    const void* bias;
    const void* residual;
    int64_t ldr;
    void* out;
    int64_t ldo;
    int32_t M, N, K, KB, epi, out_dtype, res_dtype, group_shift;
    uint32_t flags;
    float eps;
    float inv_k;     // 1 / K
    int32_t n_out;   // output columns: N, or N / 2 with SiLU*up
    int32_t units;   // 16-row units
    int32_t uq, ur;  // units / grid, units % grid: CTAs below ur own uq + 1 units, the rest uq
    int32_t nkw;     // k-blocks of the widest warp: ceil(KB / 8)
    int32_t pitch;   // bytes per staged activation row (per warp)
    int32_t upc;     // units per CTA at most (fixes the shared-memory strides)
    int32_t rbk;     // weight bytes per row (K/2, K or 2K)
    uint32_t sm_w, sm_sc, sm_x, sm_xs, sm_part, sm_misc, sm_bar;
    uint32_t sm_red;  // K split: [half][16 rows][8] partial sums + [8] sum(x^2) read by cluster rank 0
    long long wait_cycles;
};

// 1-D bulk copy global -> shared on the TMA engine, completion counted in bytes
// on an mbarrier (16-byte aligned addresses, size a multiple of 16; no multicast).
__device__ __forceinline__ void lean_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Rows of tile `tile` of unit u: 16 u (+ N/2 for the up half of SiLU*up).
__device__ __forceinline__ int lean_row(const LeanParams& p, int u, int tile) {
    return tile == 0 ? 16 * u : (p.N >> 1) + 16 * u;
}

// MR: activation rows (1 or 2), a compile-time count so the staging and its
// row reductions are straight-line code.
// KS: K slices per unit. KS > 1 (one unit per CTA, UPC 1) launches clusters of
// KS CTAs, CTA rank r of a cluster owning k-blocks [r KB/KS, (r+1) KB/KS) of the
// cluster's unit: each CTA copies only its slice of the unit's rows, and cluster
// rank 0 adds the ranks' partial sums in rank order through distributed shared
// memory before the epilogue -- for shapes with fewer 16-row units than half the
// SMs (the depth decoder's down projection: 64 units over K = 8192).
template <int FMT, int TPU, int UPC, int MR, int KS = 1>
__global__ void __launch_bounds__(kLeanThreads, 2) gemv_lean_kernel(const __grid_constant__ LeanParams p) {
    using F = Fmt3<FMT>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = lane & 3, tg = lane >> 2;
    constexpr int M = MR;
    static_assert(KS == 1 || UPC == 1, "a K-split CTA owns one unit");
    const int KB = p.KB;
    // the CTA's units and K slice, no division on the way to the weight copy
    int u0, nu, kc0, KBc;
    if constexpr (KS > 1) {
        u0 = int(blockIdx.x) / KS;
        nu = 1;
        KBc = KB / KS;
        kc0 = (int(blockIdx.x) % KS) * KBc;  // cluster rank x slice (clusters are KS consecutive CTAs)
    } else {
        u0 = int(blockIdx.x) * p.uq + min(int(blockIdx.x), p.ur);
        nu = p.uq + (int(blockIdx.x) < p.ur ? 1 : 0);  // 1 .. UPC
        kc0 = 0;
        KBc = KB;
    }
    const int kw0 = kc0 + ((warp * KBc) >> 3), nkw = kc0 + (((warp + 1) * KBc) >> 3) - kw0;  // this warp's k-blocks
    const int rbs = p.rbk / KS;  // bytes of the CTA's K slice of one row
    constexpr int RBK = FMT == BQ_W_INT4_PLAIN || FMT == BQ_W_INT4_TINYGEMM ? 64 : (FMT == BQ_W_BF16 ? 256 : 128);
    const uint32_t sbase = smem_u32(smem);
    const uint8_t* wg = static_cast<const uint8_t*>(p.w);
    const uint8_t* szg = static_cast<const uint8_t*>(p.scale);
    const bool norm = p.gamma != nullptr;

    // ---- 1. weights: one bulk copy per half (gate / up) of the CTA's contiguous rows
    const uint32_t bar_w = sbase + p.sm_bar;
    const int rows_cap = 16 * p.upc;  // rows per half in shared memory
    if (threadIdx.x == 0) {
        mbar_init(bar_w, 1);
        fence_barrier_init();
        const int half_rows = TPU == 2 ? (p.N >> 1) : p.N;
        int nrw[TPU];
        uint32_t total = 0;
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile) {
            nrw[tile] = max(min(16 * (u0 + nu), half_rows) - 16 * u0, 0);
            total += uint32_t(nrw[tile]) * uint32_t(rbs);
        }
        mbar_arrive_expect_tx(bar_w, total);
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile) {
            if (nrw[tile] == 0) continue;
            const int64_t row0 = lean_row(p, u0, tile);
            const uint32_t dst = sbase + p.sm_w + uint32_t(tile * rows_cap * rbs);
            if constexpr (KS == 1) {
                // one copy: the rows are contiguous in every layout (tinygemm: [N/8][KB][512])
                lean_bulk_g2s(dst, wg + row0 * p.rbk, uint32_t(nrw[tile]) * uint32_t(p.rbk), bar_w);
            } else if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                // the slice of each 8-row tile: KBc contiguous 512-byte k-blocks
                for (int t8 = 0; t8 < nrw[tile] / 8; ++t8)
                    lean_bulk_g2s(dst + uint32_t(t8 * KBc * 512), wg + ((row0 / 8 + t8) * KB + kc0) * 512,
                                  uint32_t(KBc * 512), bar_w);
            } else {
                for (int r = 0; r < nrw[tile]; ++r)
                    lean_bulk_g2s(dst + uint32_t(r * rbs), wg + (row0 + r) * p.rbk + int64_t(kc0) * RBK,
                                  uint32_t(rbs), bar_w);
            }
        }
    }
    if constexpr (F::kInt4) {
        // (scale, zero) of the CTA's rows for each of this warp's k-blocks: [kb][half][rows_cap] words
        for (int j = 0; j < nkw; ++j) {
            const int kb = kw0 + j;
            const int grp = (kb << 7) >> p.group_shift;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                const int half_rows = TPU == 2 ? (p.N >> 1) : p.N;
                const int nrows = min(16 * (u0 + nu), half_rows) - 16 * u0;  // a multiple of 8 (N % 8 == 0)
                const int row0 = lean_row(p, u0, tile);
                const uint32_t d = sbase + p.sm_sc + uint32_t(((kb * TPU + tile) * rows_cap) * 4);
                for (int c = lane; c < nrows / 4; c += 32)
                    cp_async16(d + c * 16, szg + (int64_t(grp) * p.N + row0) * 4 + c * 16);
            }
        }
        cp_async_commit();
    }
    __syncthreads();  // the weight barrier is initialized before anyone waits on it

    // ---- 2. static data: the epilogue's row scales and bias, gamma, zero blocks.
    // Epilogue task t = (unit ul, row r, activation row m), m fastest: m = t % M,
    // r = (t / M) % 16, ul = t / (16 M) -- compile-time divisors only.
    const int n_tasks = nu * 16 * M;
    float t_rs[2][TPU], t_rb[2][TPU];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
        const int t = threadIdx.x + kLeanThreads * i;
        const int r = (t / M) & 15, ul = t / (16 * M);
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile) {
            t_rs[i][tile] = 1.f;
            t_rb[i][tile] = 0.f;
            const int row = lean_row(p, u0 + ul, tile) + r;
            if (t < n_tasks && row < p.N) {
                if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                    float sc = static_cast<const float*>(p.scale)[row];
                    if (FMT == BQ_W_INT8 && (p.flags & BQ_FLAG_SCALE_ROUND_BF16)) sc = __bfloat162float(__float2bfloat16_rn(sc));
                    t_rs[i][tile] = sc;
                }
                if (p.bias) t_rb[i][tile] = load_act(p.bias, row, p.out_dtype);
            }
        }
    }
    const int per_row = nkw * 16;  // 16-byte chunks of one activation row in this warp's K range
    const int nch = M * per_row;
    const int nci = (nch + 31) >> 5;  // chunk rounds of the warp (uniform)
    uint4 gv[kLeanMaxChunks];
#pragma unroll
    for (int i = 0; i < kLeanMaxChunks; ++i) {
        const int t = lane + 32 * i;
        gv[i] = make_uint4(0x3F803F80u, 0x3F803F80u, 0x3F803F80u, 0x3F803F80u);  // bf16 ones
        if (norm && t < nch) {
            const int jc = t % per_row;
            gv[i] = __ldg(reinterpret_cast<const uint4*>(p.gamma + int64_t(kw0) * 128 + jc * 8));
        }
    }
    float* s_ss = reinterpret_cast<float*>(smem + p.sm_misc);  // [8 warps][8 rows] sum of x^2
    float* s_up = s_ss + 64;                                    // [8 warps][8 rows] f16 scale-back
    uint8_t* xw_ptr = smem + p.sm_x + warp * (M * p.pitch + 256);
    const uint32_t xw = sbase + p.sm_x + uint32_t(warp * (M * p.pitch + 256));
    const uint8_t* xzero = xw_ptr + M * p.pitch;  // 256 zero bytes: B fragments of rows >= M
    if (lane < 16) reinterpret_cast<uint4*>(const_cast<uint8_t*>(xzero))[lane] = make_uint4(0u, 0u, 0u, 0u);

    pdl_wait();  // x and the residual come from preceding kernels

    // ---- 3. activations of this warp's K range: registers -> gamma, sums -> staged rows
    uint4 xv[kLeanMaxChunks];
#pragma unroll
    for (int i = 0; i < kLeanMaxChunks; ++i) {
        const int t = lane + 32 * i;
        xv[i] = make_uint4(0u, 0u, 0u, 0u);
        if (i >= nci) continue;
        if (t < nch) {
            const int m = t / per_row, jc = t - m * per_row;
            xv[i] = __ldcg(reinterpret_cast<const uint4*>(p.x + m * p.ldx + int64_t(kw0) * 128 + jc * 8));
        }
    }
    float t_res[2] = {0.f, 0.f};
    if (p.epi == BQ_EPI_ADD_RESIDUAL) {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int t = threadIdx.x + kLeanThreads * i;
            const int m = t % M, r = (t / M) & 15, ul = t / (16 * M);
            const int n = 16 * (u0 + ul) + r;
            if (t < n_tasks && n < p.n_out) t_res[i] = load_act(p.residual, m * p.ldr + n, p.res_dtype);
        }
    }
    // staging: x * gamma per chunk; sum(x^2) per chunk (x itself, as RMSNorm uses it)
    float ssc[kLeanMaxChunks], xsc[kLeanMaxChunks], amc[kLeanMaxChunks];
    int mrow[kLeanMaxChunks];
#pragma unroll
    for (int i = 0; i < kLeanMaxChunks; ++i) {
        const int t = lane + 32 * i;
        mrow[i] = t < nch ? t / per_row : -1;
        ssc[i] = amc[i] = xsc[i] = 0.f;
        if (i >= nci) continue;
        const uint32_t xr[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
        const uint32_t gr[4] = {gv[i].x, gv[i].y, gv[i].z, gv[i].w};
        float ss = 0.f, am = 0.f;
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float a = bf16lo(xr[e]), b = bf16hi(xr[e]);
            ss = fmaf(a, a, ss);
            ss = fmaf(b, b, ss);
            am = fmaxf(am, fmaxf(fabsf(a * bf16lo(gr[e])), fabsf(b * bf16hi(gr[e]))));
        }
        ssc[i] = ss;
        amc[i] = am;
    }
    // per-row reductions over the warp (every lane gets each row's value)
    float row_down[MR];
#pragma unroll
    for (int m = 0; m < MR; ++m) {
        row_down[m] = 1.f;
        {
            float s = 0.f, a = 0.f;
#pragma unroll
            for (int i = 0; i < kLeanMaxChunks; ++i) {
                if (mrow[i] == m) {
                    s += ssc[i];
                    a = fmaxf(a, amc[i]);
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                s += __shfl_xor_sync(0xffffffffu, s, o);
                if constexpr (F::kF16) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
            }
            if (lane == 0) s_ss[warp * 8 + m] = s;
            if constexpr (F::kF16) {
                // f16 keeps full relative precision for any magnitude after a power-of-two shift
                int e = 0;
                if (a > 0.f && a < INFINITY) {
                    int ex;
                    frexpf(a, &ex);
                    e = min(max(ex - 15, -100), 100);
                }
                row_down[m] = __int_as_float((127 - e) << 23);
                if (lane == 0) s_up[warp * 8 + m] = __int_as_float((127 + e) << 23);
            }
        }
    }
    // rewrite as the MMA's B operand: bf16 (plain int4: pairs {0,4},{1,5},{2,6},{3,7}) or scaled f16
#pragma unroll
    for (int i = 0; i < kLeanMaxChunks; ++i) {
        if (i >= nci) break;
        const int t = lane + 32 * i;
        if (t < nch) {
            const int m = mrow[i], jc = t - m * per_row;
            const uint32_t xr[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
            const uint32_t gr[4] = {gv[i].x, gv[i].y, gv[i].z, gv[i].w};
            float v[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                v[2 * e] = bf16lo(xr[e]) * bf16lo(gr[e]);
                v[2 * e + 1] = bf16hi(xr[e]) * bf16hi(gr[e]);
            }
            uint4 o;
            if constexpr (F::kF16) {
                float dn = 1.f;
#pragma unroll
                for (int mm = 0; mm < MR; ++mm)
                    if (mm == m) dn = row_down[mm];
                o.x = pack_half2(v[0] * dn, v[1] * dn);
                o.y = pack_half2(v[2] * dn, v[3] * dn);
                o.z = pack_half2(v[4] * dn, v[5] * dn);
                o.w = pack_half2(v[6] * dn, v[7] * dn);
            } else if constexpr (FMT == BQ_W_INT4_PLAIN) {
                o.x = pack_bf162(v[0], v[4]);
                o.y = pack_bf162(v[1], v[5]);
                o.z = pack_bf162(v[2], v[6]);
                o.w = pack_bf162(v[3], v[7]);
            } else {
                o.x = pack_bf162(v[0], v[1]);
                o.y = pack_bf162(v[2], v[3]);
                o.z = pack_bf162(v[4], v[5]);
                o.w = pack_bf162(v[6], v[7]);
            }
            if constexpr (F::kInt4) {
                // the group sum X of the values the MMA sees (rounded to bf16)
                const uint32_t ov[4] = {o.x, o.y, o.z, o.w};
                float xs = 0.f;
#pragma unroll
                for (int e = 0; e < 4; ++e) xs += bf16lo(ov[e]) + bf16hi(ov[e]);
                xsc[i] = xs;
            }
            *reinterpret_cast<uint4*>(xw_ptr + m * p.pitch + jc * 16) = o;
        }
    }
    float* s_xs = reinterpret_cast<float*>(smem + p.sm_xs) + warp * (p.nkw * 8);  // [k-block][row]
    if constexpr (F::kInt4) {
        // a k-block of a row is 16 chunks held by 16 consecutive lanes (per_row is a multiple of 16)
#pragma unroll
        for (int i = 0; i < kLeanMaxChunks; ++i) {
            if (i >= nci) break;
            float v = xsc[i];
#pragma unroll
            for (int o = 8; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
            const int t = lane + 32 * i;
            if ((lane & 15) == 0 && t < nch) {
                const int m = t / per_row, jb = (t - m * per_row) >> 4;
                s_xs[jb * 8 + m] = v;
            }
        }
    }
    __syncwarp();
    // The next launch may start now: its weight copies then stream while this
    // one computes, instead of competing with this one's activation load.
    pdl_launch_dependents();
    // the weight slice (bounded wait: a timeout sets the device error bit; the
    // warp then skips its MMAs, and thread 0 waits once more so no copy is left
    // in flight when the CTA exits)
    bool w_ok = mbar_wait(bar_w, 0);
    if (F::kInt4) cp_async_wait_upto(0);
    __syncwarp();
    w_ok = __all_sync(0xffffffffu, w_ok);

    // ---- 4. main loop: k-block-major, every unit of the CTA per k-block
    constexpr int KMAGIC = F::kInt4 ? 128 + (FMT == BQ_W_INT4_TINYGEMM ? 8 : 0) : 0;
    constexpr int NCH = UPC * TPU >= 4 ? 1 : 2;  // MMA chains per unit tile (enough units interleave otherwise)
    float acc[UPC][TPU][4];
#pragma unroll
    for (int ul = 0; ul < UPC; ++ul)
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
            for (int d = 0; d < 4; ++d) acc[ul][tile][d] = 0.f;
    const uint32_t zero_blk = xw + uint32_t(M * p.pitch);
#pragma unroll 1
    for (int j = 0; j < (w_ok ? nkw : 0); ++j) {
        const int kb = kw0 + j;
        uint32_t bfr[16];
        if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
            const int m = lane & 7;
            const int koff = ((lane >> 4) * 16) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t a = m < M ? xw + uint32_t(m * p.pitch + (j * 128 + q * 32 + koff) * 2) : zero_blk;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                             : "=r"(bfr[4 * q]), "=r"(bfr[4 * q + 1]), "=r"(bfr[4 * q + 2]), "=r"(bfr[4 * q + 3])
                             : "r"(a)
                             : "memory");
            }
        } else {
            const int m = tg;
            const uint8_t* row = m < M ? xw_ptr + m * p.pitch + j * 256 : xzero;
            uint4 v[4];
            if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                v[0] = *reinterpret_cast<const uint4*>(row + (16 * tq) * 2);
                v[1] = *reinterpret_cast<const uint4*>(row + (16 * tq) * 2 + 16);
                v[2] = *reinterpret_cast<const uint4*>(row + (64 + 16 * tq) * 2);
                v[3] = *reinterpret_cast<const uint4*>(row + (64 + 16 * tq) * 2 + 16);
            } else if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                for (int h = 0; h < 4; ++h) v[h] = *reinterpret_cast<const uint4*>(row + (32 * h + 8 * tq) * 2);
            } else {
#pragma unroll
                for (int jj = 0; jj < 4; ++jj) v[jj] = *reinterpret_cast<const uint4*>(row + (32 * tq + 8 * jj) * 2);
            }
#pragma unroll
            for (int h = 0; h < 4; ++h) {
                bfr[4 * h + 0] = v[h].x;
                bfr[4 * h + 1] = v[h].y;
                bfr[4 * h + 2] = v[h].z;
                bfr[4 * h + 3] = v[h].w;
            }
        }
        float X0 = 0.f, X1 = 0.f;
        if constexpr (F::kInt4) {
            X0 = 2 * tq < M ? s_xs[j * 8 + 2 * tq] : 0.f;
            X1 = 2 * tq + 1 < M ? s_xs[j * 8 + 2 * tq + 1] : 0.f;
        }
        const int rows_cap = 16 * p.upc;
#pragma unroll
        for (int us = 0; us < UPC; ++us) {
            // One tile per unit: straight-line over UPC units (UPC is the plan's exact
            // maximum), so the compiler can overlap one unit's loads with another's
            // MMAs; a CTA with fewer units repeats its last one, and that result is
            // never written. SiLU*up (two independent tiles per unit already) keeps
            // the exit: straight-line it spills.
            if constexpr (TPU == 2) {
                if (us >= nu) break;
            }
            const int ul = us < nu ? us : nu - 1;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                // rows 16 ul + lane / 4 (r0) and + 8 (r1) of this half, the k-block's bytes
                const uint8_t* half = smem + p.sm_w + size_t(tile) * rows_cap * rbs;
                const int kbl = kb - kc0;  // k-block within the CTA's slice
                const uint8_t* src;
                int ostep;  // bytes between the two 8-row halves of the tile
                if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                    src = half + (size_t(2 * ul) * KBc + kbl) * 512 + lane * 16;  // [n8][KBc][512]
                    ostep = KBc * 512;
                } else {
                    constexpr int RB = (FMT == BQ_W_INT4_PLAIN) ? 64 : (FMT == BQ_W_BF16 ? 256 : 128);
                    src = half + size_t(16 * ul + (lane >> 2)) * rbs + kbl * RB + (lane & 3) * 16;
                    ostep = 8 * rbs;
                }
                float c2[NCH][4];
#pragma unroll
                for (int h = 0; h < NCH; ++h)
#pragma unroll
                    for (int d = 0; d < 4; ++d) c2[h][d] = 0.f;
                if constexpr (F::kInt4) {
                    const uint4 r0 = *reinterpret_cast<const uint4*>(src);
                    const uint4 r1 = *reinterpret_cast<const uint4*>(src + ostep);
                    const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                    const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
#pragma unroll
                    for (int ki = 0; ki < 8; ++ki) {
                        const uint32_t x0 = (ki & 1) ? (w0[ki >> 1] >> 8) : w0[ki >> 1];
                        const uint32_t x1 = (ki & 1) ? (w1[ki >> 1] >> 8) : w1[ki >> 1];
                        mma_bf16(c2[ki % NCH], i4_bf16(x0), i4_bf16(x1), i4_bf16(x0 >> 4), i4_bf16(x1 >> 4), bfr[2 * ki],
                                 bfr[2 * ki + 1]);
                    }
                    const uint32_t* szr = reinterpret_cast<const uint32_t*>(smem + p.sm_sc) + (kb * TPU + tile) * rows_cap + 16 * ul;
                    const uint32_t sz0 = szr[tg], sz1 = szr[tg + 8];
                    const float s0 = bf16lo(sz0), z0 = bf16hi(sz0), s1 = bf16lo(sz1), z1 = bf16hi(sz1);
                    const float A0 = float(KMAGIC) * X0, A1 = float(KMAGIC) * X1;
                    float* a = acc[us][tile];
                    float cs[4];
#pragma unroll
                    for (int d = 0; d < 4; ++d) cs[d] = NCH == 2 ? c2[0][d] + c2[NCH - 1][d] : c2[0][d];
                    a[0] += s0 * (cs[0] - A0) + z0 * X0;
                    a[1] += s0 * (cs[1] - A1) + z0 * X1;
                    a[2] += s1 * (cs[2] - A0) + z1 * X0;
                    a[3] += s1 * (cs[3] - A1) + z1 * X1;
                } else {
#pragma unroll
                    for (int b = 0; b < F::kBoxes; ++b) {
                        const uint8_t* box = src + b * 64;  // 64-byte pieces of the row's k-block
                        const uint4 r0 = *reinterpret_cast<const uint4*>(box);
                        const uint4 r1 = *reinterpret_cast<const uint4*>(box + ostep);
                        const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                        const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                        if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                            for (int e2 = 0; e2 < 2; ++e2) {
                                const int ki = 2 * b + e2;
                                mma_bf16(c2[ki % NCH], w0[2 * e2], w1[2 * e2], w0[2 * e2 + 1], w1[2 * e2 + 1], bfr[2 * ki],
                                         bfr[2 * ki + 1]);
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int ki = 4 * b + q;
                                uint32_t a0, a1, a2, a3;
                                if constexpr (FMT == BQ_W_FP8_E4M3) {
                                    a0 = e4m3x2_to_f16x2(uint16_t(w0[q] & 0xFFFF));
                                    a2 = e4m3x2_to_f16x2(uint16_t(w0[q] >> 16));
                                    a1 = e4m3x2_to_f16x2(uint16_t(w1[q] & 0xFFFF));
                                    a3 = e4m3x2_to_f16x2(uint16_t(w1[q] >> 16));
                                } else {
                                    const uint32_t x0 = w0[q] ^ 0x80808080u, x1 = w1[q] ^ 0x80808080u;
                                    a0 = i8pair_to_f16x2(x0, 0x4140u);
                                    a2 = i8pair_to_f16x2(x0, 0x4342u);
                                    a1 = i8pair_to_f16x2(x1, 0x4140u);
                                    a3 = i8pair_to_f16x2(x1, 0x4342u);
                                }
                                mma_f16(c2[ki % NCH], a0, a1, a2, a3, bfr[2 * ki], bfr[2 * ki + 1]);
                            }
                        }
                    }
#pragma unroll
                    for (int d = 0; d < 4; ++d) acc[us][tile][d] += NCH == 2 ? c2[0][d] + c2[NCH - 1][d] : c2[0][d];
                }
            }
        }
    }
    // ---- 5. warp partials [unit][tile][warp][16 rows][8 columns] (f16 formats scaled back)
    float* part = reinterpret_cast<float*>(smem + p.sm_part);
    {
        const int m0 = 2 * tq;
        float u0s = 1.f, u1s = 1.f;
        if constexpr (F::kF16) {
            u0s = m0 < M ? s_up[warp * 8 + m0] : 0.f;
            u1s = m0 + 1 < M ? s_up[warp * 8 + m0 + 1] : 0.f;
        }
#pragma unroll
        for (int ul = 0; ul < UPC; ++ul) {
            if (ul >= nu) break;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                float* pw = part + ((ul * TPU + tile) * 8 + warp) * 128;
                *reinterpret_cast<float2*>(pw + tg * 8 + m0) = make_float2(acc[ul][tile][0] * u0s, acc[ul][tile][1] * u1s);
                *reinterpret_cast<float2*>(pw + (tg + 8) * 8 + m0) =
                    make_float2(acc[ul][tile][2] * u0s, acc[ul][tile][3] * u1s);
            }
        }
    }
    __syncthreads();

    // ---- 6. epilogue: output element (row m, column n) per task, warps summed in order
    if constexpr (KS > 1) {
        // The CTA's sums over its 8 warps (in order) go to its exchange buffer;
        // cluster rank 0 adds the ranks' buffers in rank order (deterministic),
        // sum(x^2) included, and finishes the unit's outputs.
        float* red = reinterpret_cast<float*>(smem + p.sm_red);  // [TPU][16][8], then [8] sum(x^2)
        const int t = threadIdx.x;
        const int m = t % M, r = (t / M) & 15;
        if (t < n_tasks) {
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                const float* pt = part + tile * 8 * 128 + r * 8 + m;
                float a = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) a += pt[w * 128];
                red[(tile * 16 + r) * 8 + m] = a;
            }
        }
        if (t < M) {
            float a = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) a += s_ss[w * 8 + t];
            red[TPU * 128 + t] = a;
        }
        cluster_sync_all();
        if (int(blockIdx.x) % KS == 0 && t < n_tasks) {
            const uint32_t rb = smem_u32(red);
            float v[TPU];
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) v[tile] = red[(tile * 16 + r) * 8 + m];
            float ss = red[TPU * 128 + m];
#pragma unroll
            for (int q = 1; q < KS; ++q) {
                const uint32_t rq = dsmem_addr(rb, uint32_t(q));
#pragma unroll
                for (int tile = 0; tile < TPU; ++tile) v[tile] += dsmem_ld_f32(rq + uint32_t(((tile * 16 + r) * 8 + m) * 4));
                ss += dsmem_ld_f32(rq + uint32_t((TPU * 128 + m) * 4));
            }
            const float inv = norm ? rsqrtf(ss * p.inv_k + p.eps) : 1.f;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) v[tile] = v[tile] * inv * t_rs[0][tile] + t_rb[0][tile];
            const int n = 16 * u0 + r;
            if (n < p.n_out) {
                float o;
                if (p.epi == BQ_EPI_SILU_MUL)
                    o = silu(v[0]) * v[TPU - 1];
                else
                    o = p.epi == BQ_EPI_ADD_RESIDUAL ? v[0] + t_res[0] : v[0];
                store_act(p.out, m * p.ldo + n, p.out_dtype, o);
            }
        }
        // the peers' buffers stay until rank 0 has read them (its reads were consumed
        // by the stores above, so this barrier orders no memory)
        cluster_sync_relaxed();
    } else {
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const int t = threadIdx.x + kLeanThreads * i;
            if (t >= n_tasks) break;
            const int m = t % M, r = (t / M) & 15, ul = t / (16 * M);
            const int n = 16 * (u0 + ul) + r;
            float inv = 1.f;
            if (norm) {
                float a = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) a += s_ss[w * 8 + m];
                inv = rsqrtf(a * p.inv_k + p.eps);
            }
            float v[TPU];
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                const float* pt = part + (ul * TPU + tile) * 8 * 128 + r * 8 + m;
                float a = 0.f;
#pragma unroll
                for (int w = 0; w < 8; ++w) a += pt[w * 128];
                v[tile] = a * inv * t_rs[i][tile] + t_rb[i][tile];
            }
            if (n >= p.n_out) continue;
            float o;
            if (p.epi == BQ_EPI_SILU_MUL)
                o = silu(v[0]) * v[TPU - 1];
            else
                o = p.epi == BQ_EPI_ADD_RESIDUAL ? v[0] + t_res[i] : v[0];
            store_act(p.out, m * p.ldo + n, p.out_dtype, o);
        }
    }
    if (threadIdx.x == 0 && !w_ok) mbar_wait(bar_w, 0);  // no bulk copy left in flight at exit
}

}  // namespace bq
