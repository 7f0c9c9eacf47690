// bq_gemv: decode GEMV for sm_100a, weights streamed by per-warp cp.async rings.
//
//   out[m, n] = epilogue( inv[m] * sum_k (x[m,k] * gamma[k]) * W[n, k] )
//
//  * Work split: a CTA owns a contiguous range of (unit, k-block) chunks in
//    unit-major order; ranges end on unit boundaries when units are plentiful
//    ("owned", no cross-CTA reduction), otherwise the last CTA to finish a
//    unit sums its pieces. Each of the 8 warps takes a contiguous eighth of
//    the k-blocks of every unit in the range.
//  * Weights stream through a warp-private ring in shared memory, filled
//    with 16-byte cp.async copies (the load/store path): the TMA unit pays
//    ~150 cycles per box on this part, far too much for the kilobyte tiles
//    of a GEMV. The first slots are issued before the programmatic-
//    dependent-launch wait, so a dependent launch prefetches its weights
//    while the previous kernel runs; completion is tracked per warp with
//    cp.async groups, so warps never wait for each other until the final
//    reduction.
//  * A ring slot holds KPS k-blocks of up to UG units (a "unit group"), so
//    the activation fragments of a k-block are loaded once for all its units;
//    items outside the CTA's range are zero-filled and computed branch-free.
//  * Staging is row-parallel: lanes are split into row groups (32 / rows per
//    row, rounded to a power of two). int4 and bf16 weights take bf16
//    activations: one pass rewrites x*gamma as bf16 in place and accumulates
//    each lane's sum of squares. fp8 and int8 weights take f16 activations
//    scaled by a per-(warp, row) power of two from max|x*gamma|. RMSNorm's
//    1/rms is applied to the accumulator after the main loop.
//  * int4 nibbles become bf16 128 + q in registers (magic exponent 0x4300);
//    the offset is removed once per group: an MMA with an all-ones operand
//    gives each column's activation sum over the group, computed once per
//    k-block after staging and kept in shared memory.
#pragma once

#include <cuda_runtime.h>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

template <int V>
struct KConst {
    static constexpr int value = V;
};

struct Gemv3Params {
    int32_t M, N, K, KB;
    int32_t epi, group, x_dtype, out_dtype, res_dtype;
    uint32_t flags;
    float eps;
    int32_t n_half;
    int32_t tpu;         // tiles (16 rows) per unit: 1, or 2 (always 2 for SiLU*up)
    int32_t n_units;
    int32_t owned;       // 1: CTA ranges end on unit boundaries
    int32_t grid;
    int64_t total_chunks;
    int32_t ug;          // units per ring slot
    int32_t ring_slots;  // slots per consumer warp
    int32_t slot_bytes;
    int32_t nkbw;        // k-block slots per warp = ceil(KB / 8)
    int32_t p_max;       // split mode: partial slots per unit
    int32_t xrow_pitch;  // bytes per staged activation row (per warp)
    int32_t x_bulk;      // bf16 x with 16-byte aligned rows: staged with 16-byte loads
    int32_t res_bulk;    // residual rows 16-byte aligned: copied with 16-byte cp.async
    int32_t upc;         // most units any CTA covers
    int32_t group_shift; // log2(group) for int4
    int32_t ksplit;      // > 1: CTA = (unit group, K slice) rectangles; slices summed by the last arriver
    uint32_t smem_ring, smem_x, smem_xsum, smem_gamma, smem_part, smem_misc;
    const void* x;
    const void* w;
    int64_t ldx;
    const void* gamma;
    const void* scale;
    const void* bias;
    const void* residual;
    int64_t ldr;
    void* out;
    int64_t ldo;
    unsigned int* counters;
    float* partials;
};

// Misc area: floats ss[8][16], up[8][16], rowscale[4*32], rowbias[4*32],
// then 8 warps x 16 zero bytes, then the residual rows as stored in memory
// (res_dtype): [M][upc*32] elements, at most 4 bytes each.
constexpr int kMiscFixedBytes = (8 * 16 + 8 * 16 + 128 + 128) * 4 + 8 * 16;
constexpr int misc3_bytes(int upc, int rows) { return kMiscFixedBytes + upc * 32 * rows * 4; }
constexpr int kConsumerThreads = 256;
constexpr int kThreads3 = 256;
constexpr int kMaxRing = 6;  // cp.async groups a warp keeps in flight

template <int FMT>
struct Fmt3;
template <>
struct Fmt3<BQ_W_BF16> {
    static constexpr int kBoxes = 4;
    static constexpr bool kInt4 = false, kF16 = false;
};
// kF16: activations staged as f16 with a per-(warp, row) power-of-two scale
// (fp8 / int8 weights convert exactly to f16); otherwise bf16 activations
// (bf16 weights, and int4, whose codes dequantize to bf16 128 + q exactly).
template <>
struct Fmt3<BQ_W_INT4_TINYGEMM> {
    static constexpr int kBoxes = 1;
    static constexpr bool kInt4 = true, kF16 = false;
    static constexpr int kOfs = 8;
};
template <>
struct Fmt3<BQ_W_INT4_PLAIN> {
    static constexpr int kBoxes = 1;
    static constexpr bool kInt4 = true, kF16 = false;
    static constexpr int kOfs = 0;
};
template <>
struct Fmt3<BQ_W_FP8_E4M3> {
    static constexpr int kBoxes = 2;
    static constexpr bool kInt4 = false, kF16 = true;
};
template <>
struct Fmt3<BQ_W_INT8> {
    static constexpr int kBoxes = 2;
    static constexpr bool kInt4 = false, kF16 = true;
};

// Units per ring slot at most. One: every launch runs this code cold (each
// warp walks it about once per call), so instruction fetch, not arithmetic,
// is what unrolled copies of the slot body cost.
template <int MT, int TPU>
constexpr int ug_max() {
    return 1;
}

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

// Bulk prefetch of a global range into L2 (TMA unit; 16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}
__device__ __forceinline__ void prefetch_l2(const void* p) { asm volatile("prefetch.global.L2 [%0];" ::"l"(p)); }

__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
// Waits until at most n of this thread's cp.async groups are still pending.
__device__ __forceinline__ void cp_async_wait_upto(int n) {
    switch (n) {
        case 0: asm volatile("cp.async.wait_group 0;" ::: "memory"); break;
        case 1: asm volatile("cp.async.wait_group 1;" ::: "memory"); break;
        case 2: asm volatile("cp.async.wait_group 2;" ::: "memory"); break;
        case 3: asm volatile("cp.async.wait_group 3;" ::: "memory"); break;
        case 4: asm volatile("cp.async.wait_group 4;" ::: "memory"); break;
        case 5: asm volatile("cp.async.wait_group 5;" ::: "memory"); break;
        default: asm volatile("cp.async.wait_group 6;" ::: "memory"); break;
    }
}
// 16-byte copy, or 16 zero bytes when `ok` is false (src is then not read).
__device__ __forceinline__ void cp_async16_zfill(uint32_t dst, const void* src, bool ok) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(ok ? 16 : 0) : "memory");
}

// Phases of one CTA's share of a GEMV (a single launch runs them all in order).
constexpr int kPhL2 = 1;       // bulk L2 prefetch of the CTA's weight slice
constexpr int kPhPrefill = 2;  // gamma and the first ring slots (static data only)
constexpr int kPhPdl = 4;      // programmatic-dependent-launch trigger and wait
constexpr int kPhRun = 8;      // activations, staging, main loop, partials (ends in a block barrier)
constexpr int kPhEpi = 16;     // cross-warp reduction, norm factor, epilogue, stores
constexpr int kPhRing = 32;    // with kPhPrefill: also issue the first ring slots
constexpr int kPhStatic = 64;  // per-row scale / bias and zero blocks into shared memory
// The first ring slots go out before the dependent-launch wait: issuing them
// costs ~1 us of load/store-path instructions per warp, which the previous
// kernel's run hides (issued after the wait, they sit on the critical path).
constexpr int kPhAll = kPhL2 | kPhPrefill | kPhRing | kPhStatic | kPhPdl | kPhRun | kPhEpi;

struct RingState {
    int issued, ig, ij;  // ring slots issued so far; next (group, k-slot) to issue
};

// RECT: K split across CTAs (rectangles of units x a K slice; see the host
// planner). A template parameter, so kernels without it carry none of its code.
// EVEN: the host guarantees every warp an even number of k-blocks, so every ring
// slot of a one-row kernel is full and the half-slot body is not compiled.
template <int FMT, int MT, int TPU, int GPK, bool RECT = false, bool EVEN = false>
__device__ __forceinline__ void gemv_cta(const Gemv3Params& p, uint8_t* smem, const int cta, const int phases,
                                         RingState& rst) {
    using F = Fmt3<FMT>;
    constexpr int UGM = ug_max<MT, TPU>();
    constexpr int NCH = MT == 1 ? 4 : 2;  // independent MMA chains per tile
    constexpr int KPS = MT == 1 ? 2 : 1;  // k-blocks per ring slot
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int KB = p.KB, M = p.M;
    const uint32_t sbase = smem_u32(smem);
    const int RS = p.ring_slots, UG = p.ug;
    const int gpk_box = (FMT == BQ_W_INT4_TINYGEMM) ? (p.group >= 128 ? 1 : 128 / p.group) : 1;
    const int szb = F::kInt4 ? ((64 * gpk_box + 127) / 128) * 128 : 0;
    const int tile_bytes = F::kBoxes * kBoxBytes + szb;
    const bool norm = p.gamma != nullptr;

    // ---- this CTA's chunk range (32-bit: the host keeps grid * chunks < 2^32)
    uint32_t cb, ce;
    constexpr bool rect = RECT;
    int kb_lo = 0, kb_hi = KB;  // this CTA's k-blocks (a K slice in rectangle mode)
    if (rect) {
        const int ngrp = p.grid / p.ksplit, ugi = cta / p.ksplit, ks = cta - ugi * p.ksplit;
        const int u0 = int(int64_t(ugi) * p.n_units / ngrp), u1 = int(int64_t(ugi + 1) * p.n_units / ngrp);
        kb_lo = ks * KB / p.ksplit;
        kb_hi = (ks + 1) * KB / p.ksplit;
        cb = uint32_t(u0) * uint32_t(KB) + uint32_t(kb_lo);
        ce = uint32_t(u1 - 1) * uint32_t(KB) + uint32_t(kb_hi);
    } else if (p.owned) {
        cb = (uint32_t(cta) * uint32_t(p.n_units) / uint32_t(p.grid)) * uint32_t(KB);
        ce = ((uint32_t(cta) + 1) * uint32_t(p.n_units) / uint32_t(p.grid)) * uint32_t(KB);
    } else {
        const uint32_t T = uint32_t(p.total_chunks);
        cb = uint32_t(cta) * T / uint32_t(p.grid);
        ce = (uint32_t(cta) + 1) * T / uint32_t(p.grid);
    }
    const int u_first = int(cb / uint32_t(KB));
    const int u_last = int((ce - 1) / uint32_t(KB));
    const int nu = u_last - u_first + 1;  // 1..upc
    const int lo0 = int(cb - uint32_t(u_first) * KB), hi_last = int((ce - 1) - uint32_t(u_last) * KB);
    const int ngroups = (nu + UG - 1) / UG;
    auto valid = [&](int ul, int kb) {
        if (rect) return ul < nu && kb >= lo0 && kb <= hi_last;
        return ul < nu && (ul > 0 || kb >= lo0) && (ul < nu - 1 || kb <= hi_last);
    };
    auto any_valid = [&](int g, int kb) {
        bool v = false;
#pragma unroll
        for (int i = 0; i < UGM; ++i) v |= (i < UG) && valid(g * UG + i, kb);
        return v;
    };
    // this warp's k-blocks: [kw0, kw0 + nkw), a contiguous eighth of K; a ring
    // slot carries KPS consecutive ones (index jp)
    const int kw0 = kb_lo + ((warp * (kb_hi - kb_lo)) >> 3);
    const int nkw = kb_lo + (((warp + 1) * (kb_hi - kb_lo)) >> 3) - kw0;
    const int nkp = (nkw + KPS - 1) / KPS;
    auto pair_valid = [&](int g, int jp) {
        bool v = false;
#pragma unroll
        for (int kk = 0; kk < KPS; ++kk) v |= (jp * KPS + kk < nkw) && any_valid(g, kw0 + jp * KPS + kk);
        return v;
    };
    // (group, slot) issue order: advance to the next entry with work
    auto normalize = [&](int& g, int& j) {
        while (g < ngroups) {
            if (j < nkp && pair_valid(g, j)) return;
            if (j + 1 < nkp) {
                ++j;
            } else {
                j = 0;
                ++g;
            }
        }
    };
    auto tile_row = [&](int unit, int tile) -> int {
        if (p.epi == BQ_EPI_SILU_MUL) return tile == 0 ? 16 * unit : p.n_half + 16 * unit;
        return (16 * TPU) * unit + 16 * tile;
    };

    const int pitch = p.xrow_pitch;
    const uint32_t xs0 = sbase + p.smem_x;                        // [8][M * pitch + 256]
    const uint32_t gs0 = sbase + p.smem_gamma;                    // [8][nkbw][256]
    const uint32_t ring_w = sbase + p.smem_ring + warp * RS * p.slot_bytes;  // [RS][slot_bytes]

    // ---- weight copies of one ring slot (whole warp; one cp.async group)
    const uint8_t* wg = static_cast<const uint8_t*>(p.w);
    const uint8_t* szg = static_cast<const uint8_t*>(p.scale);
    // Layout of a slot: [kk][i][tile] tiles of tile_bytes. Items that are not
    // in this CTA's range (range ends, a short last group, an odd k-block
    // count) are zero-filled, so the consumer processes every item of the slot
    // without branches and they add nothing.
    auto issue = [&](int slot, int g, int jp) {
        const uint32_t dst0 = ring_w + slot * p.slot_bytes;
#pragma unroll
        for (int kk = 0; kk < KPS; ++kk)
#pragma unroll
        for (int i = 0; i < UGM; ++i) {
            if (!(i < UG)) continue;
            const int jj = jp * KPS + kk;
            const int kb = kw0 + (jj < nkw ? jj : nkw - 1);
            const bool item = jj < nkw && valid(g * UG + i, kb);
            const int unit = item ? u_first + g * UG + i : u_first;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                const int row = tile_row(unit, tile);
                const uint32_t d = dst0 + ((kk * UG + i) * TPU + tile) * tile_bytes;
                if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                    // two 8-row tiles, 512 contiguous bytes each per k-block
#pragma unroll
                    for (int q = 0; q < 2; ++q) {
                        const int pc = lane + 32 * q, nt = (row >> 3) + (pc >> 5);
                        const bool ok = item && nt * 8 < p.N;
                        cp_async16_zfill(d + pc * 16, wg + ((int64_t(ok ? nt : 0) * KB + kb) * 512 + (pc & 31) * 16), ok);
                    }
                } else {
                    // row-major: 16 rows x RB bytes per k-block, stored as 64-byte boxes [b][16][64]
                    constexpr int RB = (FMT == BQ_W_INT4_PLAIN) ? 64 : (FMT == BQ_W_BF16 ? 256 : 128);
                    const int64_t ld = (FMT == BQ_W_INT4_PLAIN) ? p.K / 2 : (FMT == BQ_W_BF16 ? int64_t(p.K) * 2 : p.K);
#pragma unroll
                    for (int q = 0; q < RB / 32; ++q) {
                        const int pc = lane + 32 * q, r = pc / (RB / 16), c = pc % (RB / 16);
                        const bool ok = item && row + r < p.N;
                        cp_async16_zfill(d + (c >> 2) * kBoxBytes + r * 64 + (c & 3) * 16,
                                         wg + (int64_t(ok ? row + r : 0) * ld + int64_t(kb) * RB + c * 16), ok);
                    }
                }
                if constexpr (F::kInt4) {
                    // scale/zero pairs of the 16 rows: 64 contiguous bytes per group
                    if (lane < 4 * gpk_box) {
                        const int gi = lane >> 2;
                        const int grp = p.group >= 128 ? (kb << 7) >> p.group_shift : kb * gpk_box + gi;
                        const bool ok = item && row + 4 * (lane & 3) < p.N;  // 4 rows per 16 bytes; N % 8 == 0
                        cp_async16_zfill(d + F::kBoxes * kBoxBytes + gi * 64 + (lane & 3) * 16,
                                         szg + ((int64_t(grp) * p.N + (ok ? row : 0)) * 4 + (lane & 3) * 16), ok);
                    }
                }
            }
        }
        cp_async_commit();
    };

    // ---- pull this CTA's whole weight slice into L2 before anything else:
    // the rings then refill from L2, not HBM, after the dependent-launch wait
    if (phases & kPhL2) {
        const int64_t row_bytes = (FMT == BQ_W_INT4_PLAIN || FMT == BQ_W_INT4_TINYGEMM)
                                      ? p.K / 2
                                      : (FMT == BQ_W_BF16 ? int64_t(p.K) * 2 : p.K);
        int r0[2], r1[2], nr = 1;
        if (p.epi == BQ_EPI_SILU_MUL) {
            r0[0] = 16 * u_first;
            r1[0] = min(p.n_half, 16 * (u_first + nu));
            r0[1] = p.n_half + 16 * u_first;
            r1[1] = min(p.N, p.n_half + 16 * (u_first + nu));
            nr = 2;
        } else {
            r0[0] = 16 * TPU * u_first;
            r1[0] = min(p.N, 16 * TPU * (u_first + nu));
        }
        if (!rect) {
            if (threadIdx.x == 0) {
                for (int q = 0; q < nr; ++q) {
                    int64_t off = int64_t(r0[q]) * row_bytes;
                    const int64_t end = int64_t(r1[q]) * row_bytes;
                    for (; off < end; off += 65536)
                        bulk_prefetch_l2(wg + off, uint32_t(end - off < 65536 ? end - off : 65536));
                }
            }
        } else {
            // the K slice of each 8-row tinygemm tile (contiguous k-blocks of 512 B), or of each row
            const int tinygemm = FMT == BQ_W_INT4_TINYGEMM;
            const int64_t kbytes = tinygemm ? 512 : row_bytes / KB;
            const int64_t len = int64_t(kb_hi - kb_lo) * kbytes;
            for (int q = 0; q < nr; ++q) {
                const int n0 = tinygemm ? r0[q] / 8 : r0[q], n1 = tinygemm ? (r1[q] + 7) / 8 : r1[q];
                for (int n = n0 + int(threadIdx.x); n < n1; n += kConsumerThreads) {
                    const int64_t off = tinygemm ? (int64_t(n) * KB + kb_lo) * 512 : int64_t(n) * row_bytes + kb_lo * kbytes;
                    for (int64_t o = 0; o < len; o += 65536)
                        bulk_prefetch_l2(wg + off + o, uint32_t(len - o < 65536 ? len - o : 65536));
                }
            }
        }
        if constexpr (F::kInt4) {
            // scale/zero rows [r0, r1) of every group row: 128-byte lines
            const int g_lo = (kb_lo * kKB) / p.group, ngrp = (kb_hi * kKB + p.group - 1) / p.group - g_lo;
            for (int q = 0; q < nr; ++q) {
                const int lines = ((r1[q] - r0[q]) * 4 + 127) / 128 + 1;
                for (int t = threadIdx.x; t < ngrp * lines; t += kConsumerThreads) {
                    const int gr = g_lo + t / lines, l = t - (t / lines) * lines;
                    const int64_t a = (int64_t(gr) * p.N + r0[q]) * 4 + l * 128;
                    if (a < (int64_t(gr) * p.N + r1[q]) * 4) prefetch_l2(szg + a);
                }
            }
        }
    }

    auto fill_ring = [&](RingState& r) {
        r.ig = 0;
        r.ij = 0;
        r.issued = 0;
        normalize(r.ig, r.ij);
        for (; r.issued < RS && r.ig < ngroups; ++r.issued) {
            issue(r.issued, r.ig, r.ij);
            if (r.ij + 1 < nkp) {
                ++r.ij;
            } else {
                r.ij = 0;
                ++r.ig;
            }
            normalize(r.ig, r.ij);
        }
    };

    // ======================================================= consumer warps
    const int tq = lane & 3, tg = lane >> 2;
    float* misc = reinterpret_cast<float*>(smem + p.smem_misc);
    float* s_ss = misc;            // [8][16]
    float* s_up = misc + 128;      // [8][16]
    float* s_rscale = misc + 256;  // [128]
    float* s_rbias = misc + 384;   // [128]
    uint8_t* s_res = reinterpret_cast<uint8_t*>(misc + 512 + 32);  // [M][upc*32] raw, after the zero blocks
    const int res_sz = p.res_dtype == BQ_DT_F32 ? 4 : 2;
    const int res_ld = p.upc * 32;
    const uint32_t zero_blk = sbase + p.smem_misc + 512 * 4 + warp * 16;
    // per-warp partial sums [upc][8 warps][TPU][MT][8 tg][nq tq][4]: only the lanes
    // whose columns 2tq, 2tq+1 can hold a real row (tq < nq = min(4, ceil(M/2)))
    float* part = reinterpret_cast<float*>(smem + p.smem_part);
    const int nq = M >= 7 ? 4 : (M + 1) >> 1;
    auto part_at = [&](int ul, int w, int tile, int mt) {
        return reinterpret_cast<float4*>(part) + (((((ul * 8 + w) * TPU + tile) * MT + mt) * 8 + tg) * nq + tq);
    };
    // per warp: M staged rows, then one zero k-block read by the B fragments of rows >= M
    uint8_t* xw_ptr = smem + p.smem_x + warp * (M * pitch + 256);
    const uint32_t xw = xs0 + warp * (M * pitch + 256);
    const uint8_t* xzero = xw_ptr + M * pitch;

    if (phases & kPhPrefill) {
        // gamma (the oldest cp.async group), then the first ring slots: all
        // static, so issued before the inputs are known to be ready
        if (norm) {
            const __nv_bfloat16* gam = static_cast<const __nv_bfloat16*>(p.gamma);
            for (int s = lane; s < nkw * 16; s += 32)
                cp_async16(gs0 + (warp * p.nkbw + (s >> 4)) * 256 + (s & 15) * 16,
                           gam + (kw0 + (s >> 4)) * 128 + (s & 15) * 8);
        }
        cp_async_commit();
        rst.ig = 0;
        rst.ij = 0;
        rst.issued = -1;  // ring not filled yet
        if (phases & kPhRing) fill_ring(rst);
    }

    // static per-call data (weights' row scales and bias, zero blocks): before the wait
    if (phases & kPhStatic) {
    if (lane < 4) reinterpret_cast<uint32_t*>(smem + p.smem_misc + 512 * 4 + warp * 16)[lane] = 0u;
    if (lane < 16) reinterpret_cast<uint4*>(const_cast<uint8_t*>(xzero))[lane] = make_uint4(0u, 0u, 0u, 0u);
    for (int r = threadIdx.x; r < nu * 32; r += kConsumerThreads) {
        const int ul = r >> 5, rr = r & 31, tile = rr >> 4;
        float sc = 1.f, bi = 0.f;
        if (tile < TPU) {
            const int n = tile_row(u_first + ul, tile) + (rr & 15);
            if (n < p.N) {
                if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                    sc = static_cast<const float*>(p.scale)[n];
                    if (FMT == BQ_W_INT8 && (p.flags & BQ_FLAG_SCALE_ROUND_BF16))
                        sc = __bfloat162float(__float2bfloat16_rn(sc));
                }
                if (p.bias) bi = load_act(p.bias, n, p.out_dtype);
            }
        }
        s_rscale[r] = sc;
        s_rbias[r] = bi;
    }

    }

    if (phases & kPhPdl) {
        pdl_wait();
    }

    if (phases & kPhRun) {
    if (rst.issued < 0) fill_ring(rst);
    int issued = rst.issued, ig = rst.ig, ij = rst.ij;
    // Inputs of this call, after the wait: x (this warp's k-blocks of every
    // row) and the residual rows go out together as two cp.async groups
    // (every thread commits both, possibly empty); only x is waited for here.
    if (p.x_bulk) {
        const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(p.x);
        const int per_row = nkw * 16, segs = M * per_row;
        for (int s = lane; s < segs; s += 32) {
            const int m = s / per_row, r = s - m * per_row;
            cp_async16(xw + m * pitch + (r >> 4) * 256 + (r & 15) * 16, xb + m * p.ldx + (kw0 + (r >> 4)) * 128 + (r & 15) * 8);
        }
    }
    cp_async_commit();
    const bool has_res = p.epi == BQ_EPI_ADD_RESIDUAL;
    if (has_res && p.res_bulk) {
        // 16-byte pieces of 16 / res_sz rows; rows past N are zero-filled
        const int per_tile = res_sz, per_row = nu * TPU * per_tile;
        const char* rb = static_cast<const char*>(p.residual);
        for (int c = threadIdx.x; c < M * per_row; c += kConsumerThreads) {
            const int m = c / per_row, r = c - m * per_row;
            const int ul = r / (TPU * per_tile), t = r - ul * (TPU * per_tile), tile = t / per_tile, q = t - tile * per_tile;
            const int n = tile_row(u_first + ul, tile) + q * (16 / res_sz);
            const int valid = min(16 / res_sz, p.N - n);
            const int lr = ul * 32 + tile * 16 + q * (16 / res_sz);
            asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(s_res) + uint32_t((m * res_ld + lr) * res_sz)),
                         "l"(rb + (int64_t(m) * p.ldr + (valid > 0 ? n : 0)) * res_sz), "r"(valid > 0 ? valid * res_sz : 0)
                         : "memory");
        }
    }
    cp_async_commit();
    if (has_res && !p.res_bulk) {
        for (int c = threadIdx.x; c < M * nu * 32; c += kConsumerThreads) {
            const int m = c / (nu * 32), lr = c - m * (nu * 32), tile = (lr & 31) >> 4;
            const int n = tile < TPU ? tile_row(u_first + (lr >> 5), tile) + (lr & 15) : p.N;
            const char* src = static_cast<const char*>(p.residual) + (int64_t(m) * p.ldr + n) * res_sz;
            uint8_t* dst = s_res + (m * res_ld + lr) * res_sz;
            if (res_sz == 4)
                *reinterpret_cast<uint32_t*>(dst) = n < p.N ? *reinterpret_cast<const uint32_t*>(src) : 0u;
            else
                *reinterpret_cast<uint16_t*>(dst) = n < p.N ? *reinterpret_cast<const uint16_t*>(src) : uint16_t(0);
        }
    }
    // groups after gamma: the first `f0` ring slots, x, residual, then refills
    const int f0 = issued;
    cp_async_wait_upto(1);  // gamma, first ring slots and x landed; the residual may be pending
    __syncwarp();
    // The next launch may start now that this one's activations have landed: its
    // prefetch then overlaps this call's compute instead of competing with the load
    // above (28-layer step, int4 M = 4 / 8 / 16: 954 / 1061 / 1325 -> 939 / 1031 / 1293 us).
    if (phases & kPhPdl) pdl_launch_dependents();

    // ---- staging: row groups of kp lanes, 16-byte units (8 values = one 8-k group)
    int lg = 0;
    while ((1 << lg) < M) ++lg;   // rows rounded up to a power of two
    const int kp_log = 5 - lg, kp = 1 << kp_log;
    const int lm = lane >> kp_log, lk = lane & (kp - 1);
    const bool rowok = lm < M;
    float ss_lane = 0.f;  // bf16 activations: this lane's share of sum(x^2), reduced after the main loop
    if constexpr (!F::kF16) {
        // One pass, no cross-lane dependency: x (times gamma) rounded to bf16 in
        // place. int4 plain pairs {s0,s4},{s1,s5},.. to match its nibble order;
        // tinygemm and bf16 weights take consecutive pairs, so with bf16 x and
        // no norm the staged row is x itself and the pass is skipped.
        const bool identity = FMT != BQ_W_INT4_PLAIN && !norm && p.x_bulk;
        const int nunits = 16 * nkw;
        const uint8_t* grow = smem + p.smem_gamma + warp * p.nkbw * 256;
        uint8_t* xrow = xw_ptr + lm * pitch;
        if (rowok && !identity) {
#pragma unroll 2
            for (int t = lk; t < nunits; t += kp) {
                const int jj = t >> 4, off = jj * 256 + (t & 15) * 16;
                float v[8];
                if (p.x_bulk) {
                    const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                    v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
                    v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
                } else {
                    const int64_t base = int64_t(lm) * p.ldx + int64_t(kw0 + jj) * 128 + (t & 15) * 8;
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = load_act(p.x, base + e, p.x_dtype);
                }
                if (norm) {
#pragma unroll
                    for (int e = 0; e < 8; ++e) ss_lane = fmaf(v[e], v[e], ss_lane);
                    const uint4 gv = *reinterpret_cast<const uint4*>(grow + off);
                    v[0] *= bf16lo(gv.x); v[1] *= bf16hi(gv.x); v[2] *= bf16lo(gv.y); v[3] *= bf16hi(gv.y);
                    v[4] *= bf16lo(gv.z); v[5] *= bf16hi(gv.z); v[6] *= bf16lo(gv.w); v[7] *= bf16hi(gv.w);
                }
                uint4 o;
                if constexpr (FMT == BQ_W_INT4_PLAIN) {
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
                *reinterpret_cast<uint4*>(xrow + off) = o;
            }
        }
    } else {
        const int nunits = 16 * nkw;
        const uint8_t* grow = smem + p.smem_gamma + warp * p.nkbw * 256;
        uint8_t* xrow = xw_ptr + lm * pitch;
        auto load8 = [&](int t, float (&v)[8]) {
            const int jj = t >> 4, off = jj * 256 + (t & 15) * 16;
            if (p.x_bulk) {
                const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
                v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
            } else {
                const int64_t base = int64_t(lm) * p.ldx + int64_t(kw0 + jj) * 128 + (t & 15) * 8;
#pragma unroll
                for (int e = 0; e < 8; ++e) v[e] = load_act(p.x, base + e, p.x_dtype);
            }
            if (norm) {
                const uint4 gv = *reinterpret_cast<const uint4*>(grow + off);
                v[0] *= bf16lo(gv.x); v[1] *= bf16hi(gv.x); v[2] *= bf16lo(gv.y); v[3] *= bf16hi(gv.y);
                v[4] *= bf16lo(gv.z); v[5] *= bf16hi(gv.z); v[6] *= bf16lo(gv.w); v[7] *= bf16hi(gv.w);
            }
        };
        // pass 1: sum of squares of x (not x*gamma) and max |x * gamma|
        float ss = 0.f, amax = 0.f;
        if (rowok) {
#pragma unroll 2
            for (int t = lk; t < nunits; t += kp) {
                const int jj = t >> 4, off = jj * 256 + (t & 15) * 16;
                float v[8];
                if (p.x_bulk) {
                    const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                    v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
                    v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
                } else {
                    const int64_t base = int64_t(lm) * p.ldx + int64_t(kw0 + jj) * 128 + (t & 15) * 8;
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = load_act(p.x, base + e, p.x_dtype);
                }
                float gg[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
                if (norm) {
                    const uint4 gv = *reinterpret_cast<const uint4*>(grow + off);
                    gg[0] = bf16lo(gv.x); gg[1] = bf16hi(gv.x); gg[2] = bf16lo(gv.y); gg[3] = bf16hi(gv.y);
                    gg[4] = bf16lo(gv.z); gg[5] = bf16hi(gv.z); gg[6] = bf16lo(gv.w); gg[7] = bf16hi(gv.w);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ss = fmaf(v[e], v[e], ss);
                    amax = fmaxf(amax, fabsf(v[e] * gg[e]));
                }
            }
        }
        for (int o = kp >> 1; o; o >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, o);
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        }
        int e = 0;
        if (amax > 0.f && amax < INFINITY) {
            int ex;
            frexpf(amax, &ex);
            e = min(max(ex - 15, -100), 100);
        }
        const float down = __int_as_float((127 - e) << 23);
        if (lk == 0 && lm < M) {
            s_ss[warp * 16 + lm] = ss;
            s_up[warp * 16 + lm] = __int_as_float((127 + e) << 23);
        }
        // pass 2: rewrite the row in place as f16 scaled by 2^-e
        if (rowok) {
#pragma unroll 2
            for (int t = lk; t < nunits; t += kp) {
                const int off = (t >> 4) * 256 + (t & 15) * 16;
                float v[8];
                load8(t, v);
                uint4 o;
                o.x = pack_half2(v[0] * down, v[1] * down);
                o.y = pack_half2(v[2] * down, v[3] * down);
                o.z = pack_half2(v[4] * down, v[5] * down);
                o.w = pack_half2(v[6] * down, v[7] * down);
                *reinterpret_cast<uint4*>(xrow + off) = o;
            }
        }
    }
    __syncwarp();

    // activation fragments (B operand) of k-slot j, per M tile
    auto load_bfrag = [&](int j, uint32_t (&bfr)[MT][16]) {
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                const int m = 8 * mt + (lane & 7);
                const int koff = ((lane >> 4) * 16) + ((lane >> 3) & 1) * 8;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const uint32_t a = m < M ? xw + m * pitch + (j * 128 + q * 32 + koff) * 2 : zero_blk;
                    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                                 : "=r"(bfr[mt][4 * q]), "=r"(bfr[mt][4 * q + 1]), "=r"(bfr[mt][4 * q + 2]),
                                   "=r"(bfr[mt][4 * q + 3])
                                 : "r"(a)
                                 : "memory");
                }
            } else {
                const int m = 8 * mt + tg;
                const uint8_t* row = m < M ? xw_ptr + m * pitch + j * 256 : xzero;
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
                    bfr[mt][4 * h + 0] = v[h].x;
                    bfr[mt][4 * h + 1] = v[h].y;
                    bfr[mt][4 * h + 2] = v[h].z;
                    bfr[mt][4 * h + 3] = v[h].w;
                }
            }
        }
    };

    // ---- int4: per-group (A, X) of columns m0, m0+1 for every k-block of this
    // warp, once: an MMA with a 0/1 indicator A operand sums the low-nibble
    // (rows 0-7) and high-nibble (rows 8-15) activations of each column.
    // Lanes tg == 0 keep {A(m0), X(m0), A(m0+1), X(m0+1)} in shared memory.
    float4* xsum4 = reinterpret_cast<float4*>(smem + p.smem_xsum) + warp * (p.nkbw * GPK * MT * 4);
    if constexpr (F::kInt4) {
#pragma unroll 2
        for (int j = 0; j < nkw; ++j) {
            uint32_t bf[MT][16];
            load_bfrag(j, bf);
#pragma unroll
            for (int sg = 0; sg < GPK; ++sg) {
                float c2[2][MT][4];
#pragma unroll
                for (int h = 0; h < 2; ++h)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int d = 0; d < 4; ++d) c2[h][mt][d] = 0.f;
#pragma unroll
                for (int ii = 0; ii < 8 / GPK; ++ii) {
                    const int i = sg * (8 / GPK) + ii;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        mma_bf16(c2[ii & 1][mt], 0x3F803F80u, 0u, 0x3F803F80u, 0u, bf[mt][2 * i], bf[mt][2 * i + 1]);
                }
                if (tg == 0) {
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        // rows 0-7 of the indicator hold sum_k x over the 16-k chunks of this group
                        const float x0 = c2[0][mt][0] + c2[1][mt][0], x1 = c2[0][mt][1] + c2[1][mt][1];
                        constexpr float kMagic = 128.f + float(F::kOfs);  // dequantized code = 128 + q
                        xsum4[((j * GPK + sg) * MT + mt) * 4 + tq] = make_float4(kMagic * x0, x0, kMagic * x1, x1);
                    }
                }
            }
        }
        __syncwarp();
    }

    // ---- main loop: unit groups, then this warp's k-slots
    int slot = 0, consumed = 0;
#pragma unroll 1
    for (int g = 0; g < ngroups; ++g) {
        float acc[UGM][TPU][MT][4];
#pragma unroll
        for (int i = 0; i < UGM; ++i)
#pragma unroll
            for (int b = 0; b < TPU; ++b)
#pragma unroll
                for (int c = 0; c < MT; ++c)
#pragma unroll
                    for (int d = 0; d < 4; ++d) acc[i][b][c][d] = 0.f;
#pragma unroll 1
        for (int jp = 0; jp < nkp; ++jp) {
            if (!pair_valid(g, jp)) continue;
            // this slot's group is complete once at most the groups issued after it are pending
            // (x and residual count for the first f0 slots)
            cp_async_wait_upto(issued - 1 - consumed + (consumed < f0 ? 2 : 0));
            __syncwarp();
            // KH = k-blocks of this slot inside the warp's range: KPS, or 1 for the last slot of a
            // warp with an odd count (e.g. K = 1024); a compile-time count keeps the full-slot body
            // free of per-k-block branches
            auto slot_body = [&](auto kh_c) {
                constexpr int KH = decltype(kh_c)::value;
                const uint8_t* src0 = smem + p.smem_ring + (warp * RS + slot) * p.slot_bytes;
                uint32_t bfr[KPS][MT][16];
                // int4: per-group (A, X) of columns m0, m0+1 from indicator MMAs
                float sA[KPS][GPK][MT][2], sX[KPS][GPK][MT][2];
#pragma unroll
                for (int kk = 0; kk < KPS; ++kk) {
                    if (kk >= KH) continue;
                    load_bfrag(jp * KPS + kk, bfr[kk]);
                }
                if constexpr (F::kInt4) {
#pragma unroll
                    for (int kk = 0; kk < KPS; ++kk) {
                        if (kk >= KH) continue;
                        const int jj = jp * KPS + kk;
#pragma unroll
                        for (int sg = 0; sg < GPK; ++sg)
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                const float4 ax = xsum4[((jj * GPK + sg) * MT + mt) * 4 + tq];
                                sA[kk][sg][mt][0] = ax.x;
                                sX[kk][sg][mt][0] = ax.y;
                                sA[kk][sg][mt][1] = ax.z;
                                sX[kk][sg][mt][1] = ax.w;
                            }
                    }
                }
#pragma unroll
                for (int i = 0; i < UGM; ++i) {
                    if (!(i < UG)) continue;
#pragma unroll
                    for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
                    for (int kk = 0; kk < KPS; ++kk) {
                        if (kk >= KH) continue;
                        const uint8_t* src = src0 + ((kk * UG + i) * TPU + tile) * tile_bytes;
                        if constexpr (F::kInt4) {
                            const uint4 r0 = *reinterpret_cast<const uint4*>(src + lane * 16);
                            const uint4 r1 = *reinterpret_cast<const uint4*>(src + 512 + lane * 16);
                            const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                            const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                            const uint8_t* szs = src + kBoxBytes;
#pragma unroll
                            for (int sg = 0; sg < GPK; ++sg) {
                                float c2[NCH][MT][4];
#pragma unroll
                                for (int h = 0; h < NCH; ++h)
#pragma unroll
                                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                        for (int d = 0; d < 4; ++d) c2[h][mt][d] = 0.f;
#pragma unroll
                                for (int ii = 0; ii < 8 / GPK; ++ii) {
                                    const int ki = sg * (8 / GPK) + ii;
                                    const uint32_t x0 = (ki & 1) ? (w0[ki >> 1] >> 8) : w0[ki >> 1];
                                    const uint32_t x1 = (ki & 1) ? (w1[ki >> 1] >> 8) : w1[ki >> 1];
                                    const uint32_t a0 = i4_bf16(x0), a2 = i4_bf16(x0 >> 4);
                                    const uint32_t a1 = i4_bf16(x1), a3 = i4_bf16(x1 >> 4);
#pragma unroll
                                    for (int mt = 0; mt < MT; ++mt)
                                        mma_bf16(c2[ii % NCH][mt], a0, a1, a2, a3, bfr[kk][mt][2 * ki], bfr[kk][mt][2 * ki + 1]);
                                }
#pragma unroll
                                for (int h = 1; h < NCH; ++h)
#pragma unroll
                                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                        for (int d = 0; d < 4; ++d) c2[0][mt][d] += c2[h][mt][d];
                                const int gi = (p.group >= 128) ? 0 : sg;
                                const uint32_t sz0 = *reinterpret_cast<const uint32_t*>(szs + gi * 64 + tg * 4);
                                const uint32_t sz1 = *reinterpret_cast<const uint32_t*>(szs + gi * 64 + (tg + 8) * 4);
                                const float s0 = bf16lo(sz0), z0 = bf16hi(sz0), s1 = bf16lo(sz1), z1 = bf16hi(sz1);
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt) {
                                    float* a = acc[i][tile][mt];
                                    a[0] += s0 * (c2[0][mt][0] - sA[kk][sg][mt][0]) + z0 * sX[kk][sg][mt][0];
                                    a[1] += s0 * (c2[0][mt][1] - sA[kk][sg][mt][1]) + z0 * sX[kk][sg][mt][1];
                                    a[2] += s1 * (c2[0][mt][2] - sA[kk][sg][mt][0]) + z1 * sX[kk][sg][mt][0];
                                    a[3] += s1 * (c2[0][mt][3] - sA[kk][sg][mt][1]) + z1 * sX[kk][sg][mt][1];
                                }
                            }
                        } else {
                            float c2[NCH][MT][4];
#pragma unroll
                            for (int h = 0; h < NCH; ++h)
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                    for (int d = 0; d < 4; ++d) c2[h][mt][d] = 0.f;
#pragma unroll
                            for (int b = 0; b < F::kBoxes; ++b) {
                                const uint8_t* box = src + b * kBoxBytes;
                                const uint4 r0 = *reinterpret_cast<const uint4*>(box + lane * 16);
                                const uint4 r1 = *reinterpret_cast<const uint4*>(box + 512 + lane * 16);
                                const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                                const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                                if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                                    for (int e2 = 0; e2 < 2; ++e2) {
                                        const int ki = 2 * b + e2;
#pragma unroll
                                        for (int mt = 0; mt < MT; ++mt)
                                            mma_bf16(c2[ki % NCH][mt], w0[2 * e2], w1[2 * e2], w0[2 * e2 + 1], w1[2 * e2 + 1],
                                                     bfr[kk][mt][2 * ki], bfr[kk][mt][2 * ki + 1]);
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
#pragma unroll
                                        for (int mt = 0; mt < MT; ++mt)
                                            mma_f16(c2[ki % NCH][mt], a0, a1, a2, a3, bfr[kk][mt][2 * ki], bfr[kk][mt][2 * ki + 1]);
                                    }
                                }
                            }
#pragma unroll
                            for (int h = 0; h < NCH; ++h)
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                                    for (int d = 0; d < 4; ++d) acc[i][tile][mt][d] += c2[h][mt][d];
                        }
                    }
                }
            };
            if constexpr (KPS == 1 || EVEN) {
                slot_body(KConst<KPS>{});
            } else {
                if (jp * KPS + KPS <= nkw)
                    slot_body(KConst<KPS>{});
                else
                    slot_body(KConst<1>{});
            }
            __syncwarp();  // every lane is done reading the slot: refill it
            ++consumed;
            if (ig < ngroups) {
                issue(slot, ig, ij);
                ++issued;
                if (ij + 1 < nkp) {
                    ++ij;
                } else {
                    ij = 0;
                    ++ig;
                }
                normalize(ig, ij);
            }
            if (++slot == RS) slot = 0;
        }
        // this group's partials, back to true scale (zeros for units this warp never saw)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int m0 = 8 * mt + 2 * tq;
            const float u0 = m0 < M ? (F::kF16 ? s_up[warp * 16 + m0] : 1.f) : 0.f;
            const float u1 = m0 + 1 < M ? (F::kF16 ? s_up[warp * 16 + m0 + 1] : 1.f) : 0.f;
#pragma unroll
            for (int i = 0; i < UGM; ++i) {
                const int ul = g * UG + i;
                if (!(i < UG && ul < nu)) continue;
#pragma unroll
                for (int tile = 0; tile < TPU; ++tile) {
                    if (tq < nq)
                        *part_at(ul, warp, tile, mt) = make_float4(acc[i][tile][mt][0] * u0, acc[i][tile][mt][1] * u1,
                                                                   acc[i][tile][mt][2] * u0, acc[i][tile][mt][3] * u1);
                }
            }
        }
    }
    if constexpr (!F::kF16) {
        if (norm) {
            for (int o = kp >> 1; o; o >>= 1) ss_lane += __shfl_xor_sync(0xffffffffu, ss_lane, o);
            if (lk == 0 && lm < M) s_ss[warp * 16 + lm] = ss_lane;
        }
    }
    if (has_res) cp_async_wait_upto(0);  // this thread's residual pieces
    __syncthreads();
    }  // kPhRun

    if (!(phases & kPhEpi)) return;
    // ---- reduce over warps, norm factor, epilogue. Task = (ul, mt).
#pragma unroll 1
    for (int task = warp; task < nu * MT; task += 8) {
        const int ul = task / MT, mt = task - (task / MT) * MT;
        const int unit = u_first + ul;
        float v[TPU][4];
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile) {
            float4 q[8];
#pragma unroll
            for (int w = 0; w < 8; ++w) q[w] = tq < nq ? *part_at(ul, w, tile, mt) : make_float4(0.f, 0.f, 0.f, 0.f);
            v[tile][0] = ((q[0].x + q[1].x) + (q[2].x + q[3].x)) + ((q[4].x + q[5].x) + (q[6].x + q[7].x));
            v[tile][1] = ((q[0].y + q[1].y) + (q[2].y + q[3].y)) + ((q[4].y + q[5].y) + (q[6].y + q[7].y));
            v[tile][2] = ((q[0].z + q[1].z) + (q[2].z + q[3].z)) + ((q[4].z + q[5].z) + (q[6].z + q[7].z));
            v[tile][3] = ((q[0].w + q[1].w) + (q[2].w + q[3].w)) + ((q[4].w + q[5].w) + (q[6].w + q[7].w));
        }
        const int m0 = 8 * mt + 2 * tq;
        const bool full = !rect && (ul > 0 || lo0 == 0) && (ul < nu - 1 || hi_last == KB - 1);
        if (!full) {
            // split mode: pieces = CTAs covering the unit, fixed summation order
            int npieces, me;
            if (rect) {
                npieces = p.ksplit;  // one piece per K slice, in slice order
                me = cta - (cta / p.ksplit) * p.ksplit;
            } else {
                const uint32_t c_first = uint32_t(unit) * KB, c_last = c_first + KB - 1;
                const uint32_t T = uint32_t(p.total_chunks);
                const int cta_f = int(((c_first + 1) * uint32_t(p.grid) - 1) / T);
                const int cta_l = int(((c_last + 1) * uint32_t(p.grid) - 1) / T);
                npieces = cta_l - cta_f + 1;
                me = cta - cta_f;
            }
            float* base = p.partials + (int64_t(unit) * p.p_max) * (TPU * 2 * 128);
            float* mine = base + int64_t(me) * (TPU * 2 * 128);
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile)
                __stcg(reinterpret_cast<float4*>(mine + ((tile * 2 + mt) * 32 + lane) * 4),
                       make_float4(v[tile][0], v[tile][1], v[tile][2], v[tile][3]));
            __threadfence();
            __syncwarp();
            unsigned int old = 0;
            if (lane == 0) old = atomicAdd(p.counters + unit * 2 + mt, 1u);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old != unsigned(npieces - 1)) continue;
            __threadfence();
            float t[TPU][4];
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
                for (int d = 0; d < 4; ++d) t[tile][d] = 0.f;
            for (int q = 0; q < npieces; ++q) {
#pragma unroll
                for (int tile = 0; tile < TPU; ++tile) {
                    float4 x4;
                    if (q == me)
                        x4 = make_float4(v[tile][0], v[tile][1], v[tile][2], v[tile][3]);
                    else
                        x4 = ldcg_f4(base + int64_t(q) * (TPU * 2 * 128) + ((tile * 2 + mt) * 32 + lane) * 4);
                    t[tile][0] += x4.x;
                    t[tile][1] += x4.y;
                    t[tile][2] += x4.z;
                    t[tile][3] += x4.w;
                }
            }
            if (lane == 0) atomicExch(p.counters + unit * 2 + mt, 0u);
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
                for (int d = 0; d < 4; ++d) v[tile][d] = t[tile][d];
        }
        float inv0 = 1.f, inv1 = 1.f;
        if (norm) {
            // lanes 0-15: row sums of squares over the 8 warps, then 1/rms per row
            float a = 0.f;
            if (lane < M) {
#pragma unroll
                for (int w = 0; w < 8; ++w) a += s_ss[w * 16 + lane];
            }
            const float invl = rsqrtf(a / float(p.K) + p.eps);
            inv0 = __shfl_sync(0xffffffffu, invl, m0 & 31);
            inv1 = __shfl_sync(0xffffffffu, invl, (m0 + 1) & 31);
        }
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int rr = tile * 16 + tg + (d >> 1) * 8;
                v[tile][d] = v[tile][d] * ((d & 1) ? inv1 : inv0) * s_rscale[ul * 32 + rr] + s_rbias[ul * 32 + rr];
            }
        if (p.epi == BQ_EPI_SILU_MUL) {
#pragma unroll
            for (int d = 0; d < 4; ++d) {
                const int n = 16 * unit + tg + (d >> 1) * 8;
                const int m = m0 + (d & 1);
                if (n < p.n_half && m < M)
                    store_act(p.out, m * p.ldo + n, p.out_dtype, silu(v[0][d]) * v[TPU - 1][d]);
            }
        } else {
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile)
#pragma unroll
                for (int d = 0; d < 4; ++d) {
                    const int rr = tile * 16 + tg + (d >> 1) * 8;
                    const int n = tile_row(unit, tile) + tg + (d >> 1) * 8;
                    const int m = m0 + (d & 1);
                    if (n < p.N && m < M) {
                        float o = v[tile][d];
                        if (p.epi == BQ_EPI_ADD_RESIDUAL) {
                            const uint8_t* q = s_res + (m * res_ld + ul * 32 + rr) * res_sz;
                            o += res_sz == 4 ? *reinterpret_cast<const float*>(q)
                                             : (p.res_dtype == BQ_DT_BF16
                                                    ? __bfloat162float(*reinterpret_cast<const __nv_bfloat16*>(q))
                                                    : __half2float(*reinterpret_cast<const __half*>(q)));
                        }
                        store_act(p.out, m * p.ldo + n, p.out_dtype, o);
                    }
                }
        }
    }
}

template <int FMT, int MT, int TPU, int GPK, bool RECT = false, bool EVEN = false>
__global__ void __launch_bounds__(kThreads3, 2) gemv3_kernel(const Gemv3Params p) {
    extern __shared__ __align__(1024) uint8_t smem[];
    RingState rst;
    gemv_cta<FMT, MT, TPU, GPK, RECT, EVEN>(p, smem, int(blockIdx.x), kPhAll, rst);
}

// Host: kernel parameters of one launch from a descriptor and its plan.
void fill_gemv3_params(const bq_gemv_desc* d, const Gemv3Plan& pl, int row0, void* workspace, Gemv3Params* out);

}  // namespace bq
