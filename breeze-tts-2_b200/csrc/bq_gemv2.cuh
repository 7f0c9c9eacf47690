// bq_gemv v2: CTA-owned output units, warps split K inside the CTA.
//
//   out[m, n] = epilogue( inv[m] * sum_k (x[m,k] * gamma[k]) * W[n, k] )
//
//  * Work: a CTA gets a contiguous range of chunks (unit, k-block) in
//    unit-major order. When there are at least as many units as CTAs the
//    ranges end on unit boundaries ("owned": no cross-CTA reduction at all);
//    otherwise a unit can be split between CTAs and the last CTA to finish it
//    sums the pieces (arrival counter in a workspace, fixed order).
//  * Inside a CTA, warp w handles the k-blocks kb = w (mod 8) of every unit
//    in the range and stages only the activations of those k-blocks, in
//    natural order, in its own shared-memory rows: no block barrier before
//    the tensor-core loop. RMSNorm is applied as a per-row factor on the
//    accumulator (sum of squares reduced at the single block barrier).
//  * Weights stream through a per-warp ring of TMA tile loads issued before
//    the programmatic-dependent-launch wait; when the CTA's share fits, the
//    ring holds all of it, so a dependent launch prefetches its weights
//    while the previous kernel is still running. gamma is prefetched the
//    same way; per-row scale and bias are read before the wait and the
//    residual right after it, so the epilogue does no global loads.
//  * The code is kept compact (one chunk body reused by a rolled loop): this
//    kernel is latency-bound and every warp walks its code about once, so
//    instruction fetch, not arithmetic, is what unrolled variants pay for.
#pragma once

#include <cuda_runtime.h>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

struct Gemv2Params {
    int32_t M, N, K, KB;
    int32_t epi, group, x_dtype, out_dtype, res_dtype;
    uint32_t flags;
    float eps;
    int32_t n_half;
    int32_t tpu;        // tiles (16 rows) per unit: 1, or 2 (always 2 for SiLU*up)
    int32_t n_units;
    int32_t owned;      // 1: CTA ranges end on unit boundaries
    int32_t grid;
    int64_t total_chunks;
    int32_t ring_slots, slot_bytes, nkbw;  // nkbw = k-blocks per warp = ceil(KB / 8)
    int32_t p_max;      // split mode: partial slots per unit
    int32_t xrow_pitch; // bytes per staged activation row (per warp)
    int32_t x_vec;      // bf16 x, rows 8-byte aligned: asynchronous staging
    int32_t upc;        // most units any CTA covers
    int32_t group_shift; // log2(group) for int4
    uint32_t smem_bars, smem_ring, smem_x, smem_xsum, smem_gamma, smem_part, smem_misc;
    const void* x;
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

// Misc area (floats): ss[8][16], up[8][16], rowscale[4*32], rowbias[4*32],
// res[4*32][16], then 8 warps x 16 zero bytes.
constexpr int kMiscBytes = (8 * 16 + 8 * 16 + 128 + 128 + 128 * 16) * 4 + 8 * 16;

template <int FMT>
struct Fmt2;
template <>
struct Fmt2<BQ_W_BF16> {
    static constexpr int kBoxes = 4;
    static constexpr bool kInt4 = false, kF16 = false;
};
template <>
struct Fmt2<BQ_W_INT4_TINYGEMM> {
    static constexpr int kBoxes = 1;
    static constexpr bool kInt4 = true, kF16 = true;
    static constexpr int kOfs = 8;
};
template <>
struct Fmt2<BQ_W_INT4_PLAIN> {
    static constexpr int kBoxes = 1;
    static constexpr bool kInt4 = true, kF16 = true;
    static constexpr int kOfs = 0;
};
template <>
struct Fmt2<BQ_W_FP8_E4M3> {
    static constexpr int kBoxes = 2;
    static constexpr bool kInt4 = false, kF16 = true;
};
template <>
struct Fmt2<BQ_W_INT8> {
    static constexpr int kBoxes = 2;
    static constexpr bool kInt4 = false, kF16 = true;
};

__device__ __forceinline__ float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

template <int FMT, int MT, int TPU, int GPK>
__global__ void __launch_bounds__(256, 2)
    gemv2_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_sz,
                 const Gemv2Params p) {
    using F = Fmt2<FMT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = lane & 3, tg = lane >> 2;
    const int KB = p.KB, M = p.M;
    const uint32_t sbase = smem_u32(smem);
    const int RS = p.ring_slots;
    const int gpk_box = (FMT == BQ_W_INT4_TINYGEMM) ? (p.group >= 128 ? 1 : 128 / p.group) : 1;
    const int szb = F::kInt4 ? ((64 * gpk_box + 127) / 128) * 128 : 0;
    const uint32_t tx_bytes = TPU * F::kBoxes * kBoxBytes + (F::kInt4 ? TPU * 64 * gpk_box : 0);

    // ---- this CTA's chunk range and units (32-bit arithmetic: the host keeps
    // grid * total_chunks below 2^32)
    uint32_t cb, ce;
    if (p.owned) {
        cb = (blockIdx.x * uint32_t(p.n_units) / uint32_t(p.grid)) * uint32_t(KB);
        ce = ((blockIdx.x + 1) * uint32_t(p.n_units) / uint32_t(p.grid)) * uint32_t(KB);
    } else {
        const uint32_t T = uint32_t(p.total_chunks);
        cb = blockIdx.x * T / uint32_t(p.grid);
        ce = (blockIdx.x + 1) * T / uint32_t(p.grid);
    }
    const int u_first = int(cb / uint32_t(KB));
    const int u_last = int((ce - 1) / uint32_t(KB));
    const int nu = u_last - u_first + 1;  // 1..upc (host guarantees)
    const int lo0 = int(cb - uint32_t(u_first) * KB), hi_last = int((ce - 1) - uint32_t(u_last) * KB);
    auto unit_lo = [&](int ul) { return ul == 0 ? lo0 : 0; };
    auto unit_hi = [&](int ul) { return ul == nu - 1 ? hi_last : KB - 1; };
    auto in_span = [&](int kb) {
        if (nu >= 3) return true;
        if (nu == 2) return kb >= lo0 || kb <= hi_last;
        return kb >= lo0 && kb <= hi_last;
    };
    auto first_kb = [&](int ul) {
        const int lo = unit_lo(ul);
        return lo + ((warp - lo) % 8 + 8) % 8;
    };
    auto tile_row = [&](int unit, int tile) -> int {
        if (p.epi == BQ_EPI_SILU_MUL) return tile == 0 ? 16 * unit : p.n_half + 16 * unit;
        return (16 * TPU) * unit + 16 * tile;
    };

    const uint32_t my_bars = sbase + p.smem_bars + warp * RS * 8;
    const uint32_t my_ring = sbase + p.smem_ring + warp * RS * p.slot_bytes;

    // ---- TMA issue over this warp's chunk sequence (lane 0 only)
    int is_ul = 0, is_kb = first_kb(0), issued = 0, is_slot = 0;
    auto issue_next = [&]() {
        while (is_ul < nu && is_kb > unit_hi(is_ul)) {
            ++is_ul;
            if (is_ul < nu) is_kb = first_kb(is_ul);
        }
        if (is_ul >= nu) return;
        const int unit = u_first + is_ul, kb = is_kb;
        const int slot = is_slot;
        is_slot = is_slot + 1 == RS ? 0 : is_slot + 1;
        const uint32_t bar = my_bars + slot * 8;
        const uint32_t dst = my_ring + slot * p.slot_bytes;
        mbar_arrive_expect_tx(bar, tx_bytes);
        for (int tile = 0; tile < TPU; ++tile) {
            const int row = tile_row(unit, tile);
#pragma unroll
            for (int b = 0; b < F::kBoxes; ++b) {
                const uint32_t d = dst + (tile * F::kBoxes + b) * kBoxBytes;
                if constexpr (FMT == BQ_W_INT4_TINYGEMM)
                    tma_load_2d(d, &tm_w, kb * 128, row >> 3, bar);
                else if constexpr (FMT == BQ_W_INT4_PLAIN)
                    tma_load_2d(d, &tm_w, kb * 64, row, bar);
                else if constexpr (FMT == BQ_W_BF16)
                    tma_load_2d(d, &tm_w, kb * 128 + 32 * b, row, bar);
                else
                    tma_load_2d(d, &tm_w, kb * 128 + 64 * b, row, bar);
            }
            if constexpr (F::kInt4) {
                const int grp = p.group >= 128 ? (kb << 7) >> p.group_shift : kb * gpk_box;
                tma_load_2d(dst + TPU * F::kBoxes * kBoxBytes + tile * szb, &tm_sz, 2 * row, grp, bar);
            }
        }
        ++issued;
        is_kb += 8;
    };
    if (lane == 0) {
        for (int s = 0; s < RS; ++s) mbar_init(my_bars + s * 8, 1);
        fence_barrier_init();
        for (int s = 0; s < RS; ++s) issue_next();
    }
    __syncwarp();

    float* misc = reinterpret_cast<float*>(smem + p.smem_misc);
    float* s_ss = misc;            // [8][16]
    float* s_up = misc + 128;      // [8][16]
    float* s_rscale = misc + 256;  // [128]
    float* s_rbias = misc + 384;   // [128]
    float* s_res = misc + 512;     // [128][16]
    const uint32_t zero_blk = sbase + p.smem_misc + (512 + 128 * 16) * 4 + warp * 16;
    if (lane < 4) reinterpret_cast<uint32_t*>(smem + p.smem_misc + (512 + 128 * 16) * 4 + warp * 16)[lane] = 0u;

    // static operands: gamma for this warp's k-blocks, per-row scale and bias
    const bool norm = p.gamma != nullptr;
    const __nv_bfloat16* gamma = static_cast<const __nv_bfloat16*>(p.gamma);
    const uint32_t gw = sbase + p.smem_gamma + warp * p.nkbw * 256;
    const uint8_t* gw_ptr = smem + p.smem_gamma + warp * p.nkbw * 256;
    if (norm) {
        for (int kb = warp, j = 0; kb < KB; kb += 8, ++j)
            cp_async8(gw + j * 256 + lane * 8, gamma + kb * 128 + lane * 4);
    }
    for (int r = threadIdx.x; r < nu * 32; r += blockDim.x) {
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

    pdl_launch_dependents();
    pdl_wait();

    // ---- activations of this warp's k-blocks (natural order, per row)
    uint8_t* xw_ptr = smem + p.smem_x + warp * (M * p.xrow_pitch);
    const uint32_t xw = sbase + p.smem_x + warp * (M * p.xrow_pitch);
    float* xsum = reinterpret_cast<float*>(smem + p.smem_xsum) + warp * (p.nkbw * GPK * 32);  // [j][sg][m][A, X]
    // per-warp zero row: B fragments of activation rows >= M read it
    const uint8_t* xzero = smem + p.smem_x + 8 * (M * p.xrow_pitch) + warp * p.xrow_pitch;
    const bool fast = p.x_vec && (p.owned || !norm);  // every k-block needed is staged
    if (fast) {
        const __nv_bfloat16* xb = static_cast<const __nv_bfloat16*>(p.x);
        for (int m = 0; m < M; ++m)
            for (int kb = warp, j = 0; kb < KB; kb += 8, ++j)
                if (in_span(kb)) cp_async8(xw + m * p.xrow_pitch + j * 256 + lane * 8, xb + m * p.ldx + kb * 128 + lane * 4);
    }
    // residual rows of the CTA's outputs (consumed in the epilogue)
    if (p.epi == BQ_EPI_ADD_RESIDUAL) {
        for (int r = threadIdx.x; r < nu * 32; r += blockDim.x) {
            const int ul = r >> 5, rr = r & 31, tile = rr >> 4;
            const int n = tile < TPU ? tile_row(u_first + ul, tile) + (rr & 15) : p.N;
            for (int m = 0; m < M; ++m) s_res[r * 16 + m] = n < p.N ? load_act(p.residual, m * p.ldr + n, p.res_dtype) : 0.f;
        }
    }
    cp_async_wait_all();
    __syncwarp();
    {
#pragma unroll 1
        for (int m = 0; m < M; ++m) {
            // pass 1: sum of squares (all k) and max |x * gamma| (staged k)
            float ss = 0.f, amax = 0.f;
#pragma unroll 1
            for (int kb = warp, j = 0; kb < KB; kb += 8, ++j) {
                const bool staged = in_span(kb);
                if (!staged && (fast || !norm)) continue;
                float v[4];
                if (fast) {
                    const uint2 raw = *reinterpret_cast<const uint2*>(xw_ptr + m * p.xrow_pitch + j * 256 + lane * 8);
                    v[0] = bf_lo(raw.x);
                    v[1] = bf_hi(raw.x);
                    v[2] = bf_lo(raw.y);
                    v[3] = bf_hi(raw.y);
                } else {
#pragma unroll
                    for (int e = 0; e < 4; ++e) v[e] = load_act(p.x, m * p.ldx + kb * 128 + lane * 4 + e, p.x_dtype);
                }
                float g[4] = {1.f, 1.f, 1.f, 1.f};
                if (norm) {
                    const uint2 gv = *reinterpret_cast<const uint2*>(gw_ptr + j * 256 + lane * 8);
                    g[0] = bf_lo(gv.x);
                    g[1] = bf_hi(gv.x);
                    g[2] = bf_lo(gv.y);
                    g[3] = bf_hi(gv.y);
                }
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    ss = fmaf(v[e], v[e], ss);
                    if (staged) amax = fmaxf(amax, fabsf(v[e] * g[e]));
                }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
                ss += __shfl_xor_sync(0xffffffffu, ss, o);
                amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            }
            int e = 0;
            if (F::kF16 && amax > 0.f && amax < INFINITY) {
                int ex;
                frexpf(amax, &ex);
                e = min(max(ex - 15, -100), 100);
            }
            const float down = __int_as_float((127 - e) << 23);
            if (lane == 0) {
                s_ss[warp * 16 + m] = ss;
                s_up[warp * 16 + m] = __int_as_float((127 + e) << 23);
            }
            // pass 2: x * gamma * 2^-e -> f16 (bf16 for bf16 weights), in place
#pragma unroll 1
            for (int kb = warp, j = 0; kb < KB; kb += 8, ++j) {
                if (!in_span(kb)) continue;
                float v[4];
                uint8_t* dst = xw_ptr + m * p.xrow_pitch + j * 256 + lane * 8;
                if (fast) {
                    const uint2 raw = *reinterpret_cast<const uint2*>(dst);
                    v[0] = bf_lo(raw.x);
                    v[1] = bf_hi(raw.x);
                    v[2] = bf_lo(raw.y);
                    v[3] = bf_hi(raw.y);
                } else {
#pragma unroll
                    for (int q = 0; q < 4; ++q) v[q] = load_act(p.x, m * p.ldx + kb * 128 + lane * 4 + q, p.x_dtype);
                }
                if (norm) {
                    const uint2 gv = *reinterpret_cast<const uint2*>(gw_ptr + j * 256 + lane * 8);
                    v[0] *= bf_lo(gv.x);
                    v[1] *= bf_hi(gv.x);
                    v[2] *= bf_lo(gv.y);
                    v[3] *= bf_hi(gv.y);
                }
                uint2 packed;
                if constexpr (F::kInt4) {
                    // values that meet high-nibble operand lanes are pre-scaled
                    // by 1/16: tinygemm k % 16 >= 8 (lanes with bit 1 set),
                    // plain layout odd k
                    float sc[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const bool hiq = (FMT == BQ_W_INT4_TINYGEMM) ? ((lane & 2) != 0) : ((q & 1) != 0);
                        sc[q] = hiq ? down * 0.0625f : down;
                    }
                    const __half2 h0 = __floats2half2_rn(v[0] * sc[0], v[1] * sc[1]);
                    const __half2 h1 = __floats2half2_rn(v[2] * sc[2], v[3] * sc[3]);
                    uint32_t u0 = *reinterpret_cast<const uint32_t*>(&h0), u1 = *reinterpret_cast<const uint32_t*>(&h1);
                    if constexpr (FMT == BQ_W_INT4_PLAIN) {
                        // pair order inside each 8-k group: {s0,s4},{s1,s5},{s2,s6},{s3,s7}
                        const bool even = (lane & 1) == 0;
                        const uint32_t partner = __shfl_xor_sync(0xffffffffu, even ? u1 : u0, 1);
                        if (even) {
                            packed.x = prmt(u0, partner, 0x5410u);
                            packed.y = prmt(u0, partner, 0x7632u);
                        } else {
                            packed.x = prmt(partner, u1, 0x5410u);
                            packed.y = prmt(partner, u1, 0x7632u);
                        }
                    } else {
                        packed.x = u0;
                        packed.y = u1;
                    }
                } else if constexpr (F::kF16) {
                    const __half2 h0 = __floats2half2_rn(v[0] * down, v[1] * down);
                    const __half2 h1 = __floats2half2_rn(v[2] * down, v[3] * down);
                    packed.x = *reinterpret_cast<const uint32_t*>(&h0);
                    packed.y = *reinterpret_cast<const uint32_t*>(&h1);
                } else {
                    packed.x = pack_bf162(v[0], v[1]);
                    packed.y = pack_bf162(v[2], v[3]);
                }
                *reinterpret_cast<uint2*>(dst) = packed;
            }
        }
    }
    for (int b = lane * 16; b < p.xrow_pitch; b += 32 * 16)
        *reinterpret_cast<uint4*>(const_cast<uint8_t*>(xzero) + b) = make_uint4(0u, 0u, 0u, 0u);
    __syncwarp();

    // activation fragments (B operand) of k-block slot j, per M tile
    auto load_bfrag = [&](int j, uint32_t (&bfr)[MT][16]) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                    const int m = 8 * mt + (lane & 7);
                    const int koff = ((lane >> 4) * 16) + ((lane >> 3) & 1) * 8;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const uint32_t a = m < M ? xw + m * p.xrow_pitch + (j * 128 + q * 32 + koff) * 2 : zero_blk;
                        asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                                     : "=r"(bfr[mt][4 * q]), "=r"(bfr[mt][4 * q + 1]), "=r"(bfr[mt][4 * q + 2]),
                                       "=r"(bfr[mt][4 * q + 3])
                                     : "r"(a)
                                     : "memory");
                    }
                } else {
                    const int m = 8 * mt + tg;
                    const uint8_t* row = (m < M ? xw_ptr + m * p.xrow_pitch : xzero) + j * 256;
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
                    for (int h = 0; h < 4; ++h) {  // plain int4 is staged in {s, s+4} pair order
                        bfr[mt][4 * h + 0] = v[h].x;
                        bfr[mt][4 * h + 1] = v[h].y;
                        bfr[mt][4 * h + 2] = v[h].z;
                        bfr[mt][4 * h + 3] = v[h].w;
                    }
                }
            }
    };

    // int4: per-group activation sums on the tensor cores. A is a 0/1
    // indicator: rows 0-7 pick the k positions that meet low-nibble operand
    // lanes, rows 8-15 the high-nibble ones, so C[0..7][m] = S_lo(m) and
    // C[8..15][m] = S_hi(m) in exactly the lanes that later need them.
    if constexpr (F::kInt4) {
#pragma unroll 1
        for (int kb = warp, j = 0; kb < KB; kb += 8, ++j) {
            if (!in_span(kb)) continue;
            uint32_t bfr[MT][16];
            load_bfrag(j, bfr);
#pragma unroll
            for (int sg = 0; sg < GPK; ++sg) {
                float c[MT][4];
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int d = 0; d < 4; ++d) c[mt][d] = 0.f;
#pragma unroll
                for (int ii = 0; ii < 8 / GPK; ++ii) {
                    const int i = sg * (8 / GPK) + ii;
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
                        mma_f16(c[mt], 0x3C003C00u, 0u, 0u, 0x3C003C00u, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                }
                if (tg == 0) {
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const int m0 = 8 * mt + 2 * tq;
                        float* xs = xsum + ((j * GPK + sg) * 16 + m0) * 2;
                        // lane (tg=0) holds c0/c1 = S_lo(m0, m0+1) (row 0), c2/c3 = S_hi (row 8)
                        const float slo0 = c[mt][0], slo1 = c[mt][1], shi0 = c[mt][2], shi1 = c[mt][3];
                        xs[0] = 1024.f * (slo0 + shi0) + float(F::kOfs) * (slo0 + 16.f * shi0);
                        xs[1] = slo0 + 16.f * shi0;
                        xs[2] = 1024.f * (slo1 + shi1) + float(F::kOfs) * (slo1 + 16.f * shi1);
                        xs[3] = slo1 + 16.f * shi1;
                    }
                }
            }
        }
        __syncwarp();
    }

    // ---- main loop: one chunk body, rolled over this warp's chunks
    const uint8_t* ring_ptr = smem + p.smem_ring + warp * RS * p.slot_bytes;
    float* part = reinterpret_cast<float*>(smem + p.smem_part);  // [upc][8 warps][TPU][MT][32][4]
    int consumed = 0, slot = 0;
    uint32_t phase = 0;
    bool failed = false;
#pragma unroll 1
    for (int ul = 0; ul < nu; ++ul) {
        float acc[TPU][MT][4];
#pragma unroll
        for (int b = 0; b < TPU; ++b)
#pragma unroll
            for (int c = 0; c < MT; ++c)
#pragma unroll
                for (int d = 0; d < 4; ++d) acc[b][c][d] = 0.f;
        const int hi = unit_hi(ul);
#pragma unroll 1
        for (int kb = first_kb(ul); kb <= hi && !failed; kb += 8) {
            if (!mbar_wait(my_bars + slot * 8, phase)) {
                failed = true;
                break;
            }
            const int j = (kb - warp) >> 3;
            const uint8_t* src = ring_ptr + slot * p.slot_bytes;
            // activation fragments of this k-block, per M tile
            uint32_t bfr[MT][16];
            load_bfrag(j, bfr);
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                if constexpr (F::kInt4) {
                    const uint4 r0 = *reinterpret_cast<const uint4*>(src + tile * kBoxBytes + lane * 16);
                    const uint4 r1 = *reinterpret_cast<const uint4*>(src + tile * kBoxBytes + 512 + lane * 16);
                    const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                    const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                    const uint8_t* szs = src + TPU * kBoxBytes + tile * szb;
#pragma unroll
                    for (int sg = 0; sg < GPK; ++sg) {
                        float ce[MT][4], co[MT][4];
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int d = 0; d < 4; ++d) ce[mt][d] = co[mt][d] = 0.f;
#pragma unroll
                        for (int ii = 0; ii < 8 / GPK; ++ii) {
                            const int i = sg * (8 / GPK) + ii;
                            const uint32_t x0 = (i & 1) ? (w0[i >> 1] >> 8) : w0[i >> 1];
                            const uint32_t x1 = (i & 1) ? (w1[i >> 1] >> 8) : w1[i >> 1];
                            const uint32_t a0 = i4lo_raw(x0);
                            const uint32_t a2 = i4hi_raw(x0);
                            const uint32_t a1 = i4lo_raw(x1);
                            const uint32_t a3 = i4hi_raw(x1);
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt) {
                                if (ii & 1)
                                    mma_f16(co[mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                                else
                                    mma_f16(ce[mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                            }
                        }
                        const int gi = (p.group >= 128) ? 0 : sg;
                        const uint32_t sz0 = *reinterpret_cast<const uint32_t*>(szs + gi * 64 + tg * 4);
                        const uint32_t sz1 = *reinterpret_cast<const uint32_t*>(szs + gi * 64 + (tg + 8) * 4);
                        const float s0 = bf_lo(sz0), z0 = bf_hi(sz0), s1 = bf_lo(sz1), z1 = bf_hi(sz1);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            // (A, X) of rows m0, m0+1: A removes the magic offsets, X is the plain sum
                            const int m0 = 8 * mt + 2 * tq;
                            const float4 ax = *reinterpret_cast<const float4*>(xsum + ((j * GPK + sg) * 16 + m0) * 2);
                            acc[tile][mt][0] += s0 * ((ce[mt][0] + co[mt][0]) - ax.x) + z0 * ax.y;
                            acc[tile][mt][1] += s0 * ((ce[mt][1] + co[mt][1]) - ax.z) + z0 * ax.w;
                            acc[tile][mt][2] += s1 * ((ce[mt][2] + co[mt][2]) - ax.x) + z1 * ax.y;
                            acc[tile][mt][3] += s1 * ((ce[mt][3] + co[mt][3]) - ax.z) + z1 * ax.w;
                        }
                    }
                } else {
                    float ce[MT][4], co[MT][4];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int d = 0; d < 4; ++d) ce[mt][d] = co[mt][d] = 0.f;
#pragma unroll
                    for (int b = 0; b < F::kBoxes; ++b) {
                        const uint8_t* box = src + (tile * F::kBoxes + b) * kBoxBytes;
                        const uint4 r0 = *reinterpret_cast<const uint4*>(box + lane * 16);
                        const uint4 r1 = *reinterpret_cast<const uint4*>(box + 512 + lane * 16);
                        const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                        const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                        if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                            for (int e = 0; e < 2; ++e) {
                                const int i = 2 * b + e;
#pragma unroll
                                for (int mt = 0; mt < MT; ++mt) {
                                    if (e & 1)
                                        mma_bf16(co[mt], w0[2 * e], w1[2 * e], w0[2 * e + 1], w1[2 * e + 1],
                                                 bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                                    else
                                        mma_bf16(ce[mt], w0[2 * e], w1[2 * e], w0[2 * e + 1], w1[2 * e + 1],
                                                 bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                                }
                            }
                        } else {
#pragma unroll
                            for (int q = 0; q < 4; ++q) {
                                const int i = 4 * b + q;
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
                                for (int mt = 0; mt < MT; ++mt) {
                                    if (q & 1)
                                        mma_f16(co[mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                                    else
                                        mma_f16(ce[mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                                }
                            }
                        }
                    }
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int d = 0; d < 4; ++d) acc[tile][mt][d] += ce[mt][d] + co[mt][d];
                }
            }
            __syncwarp();
            ++consumed;
            if (++slot == RS) {
                slot = 0;
                phase ^= 1u;
            }
            if (lane == 0 && is_ul < nu) {
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                issue_next();
            }
        }
        // this unit's partial, back to true scale
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int m0 = 8 * mt + 2 * tq;
            const float u0 = m0 < M ? s_up[warp * 16 + m0] : 0.f;
            const float u1 = m0 + 1 < M ? s_up[warp * 16 + m0 + 1] : 0.f;
#pragma unroll
            for (int tile = 0; tile < TPU; ++tile) {
                float4 v = make_float4(acc[tile][mt][0] * u0, acc[tile][mt][1] * u1, acc[tile][mt][2] * u0,
                                       acc[tile][mt][3] * u1);
                if (failed) v = make_float4(0.f, 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(part + ((((ul * 8 + warp) * TPU + tile) * MT + mt) * 32 + lane) * 4) = v;
            }
        }
    }
    if (failed) {
        // gave up on chunk `consumed`: let this warp's other copies in flight land
        const int n_issued = __shfl_sync(0xffffffffu, issued, 0);
        int s2 = slot;
        uint32_t ph2 = phase;
        for (int q = consumed; q < n_issued; ++q) {
            if (q > consumed) mbar_wait(my_bars + s2 * 8, ph2);
            if (++s2 == RS) {
                s2 = 0;
                ph2 ^= 1u;
            }
        }
    }
    __syncthreads();

    // ---- reduce over warps, norm factor, epilogue. Task = (ul, mt).
#pragma unroll 1
    for (int task = warp; task < nu * MT; task += 8) {
        const int ul = task / MT, mt = task % MT;
        const int unit = u_first + ul;
        float v[TPU][4];
#pragma unroll
        for (int tile = 0; tile < TPU; ++tile) {
#pragma unroll
            for (int d = 0; d < 4; ++d) v[tile][d] = 0.f;
#pragma unroll
            for (int w = 0; w < 8; ++w) {
                const float4 q = *reinterpret_cast<const float4*>(part + ((((ul * 8 + w) * TPU + tile) * MT + mt) * 32 + lane) * 4);
                v[tile][0] += q.x;
                v[tile][1] += q.y;
                v[tile][2] += q.z;
                v[tile][3] += q.w;
            }
        }
        const int m0 = 8 * mt + 2 * tq;
        const bool full = unit_lo(ul) == 0 && unit_hi(ul) == KB - 1;
        if (!full) {
            // split mode: pieces = CTAs covering the unit, fixed summation order
            const uint32_t c_first = uint32_t(unit) * KB, c_last = c_first + KB - 1;
            const uint32_t T = uint32_t(p.total_chunks);
            const int cta_f = int(((c_first + 1) * uint32_t(p.grid) - 1) / T);
            const int cta_l = int(((c_last + 1) * uint32_t(p.grid) - 1) / T);
            const int npieces = cta_l - cta_f + 1;
            const int me = int(blockIdx.x) - cta_f;
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
            float a0 = 0.f, a1 = 0.f;
            for (int w = 0; w < 8; ++w) {
                if (m0 < M) a0 += s_ss[w * 16 + m0];
                if (m0 + 1 < M) a1 += s_ss[w * 16 + m0 + 1];
            }
            inv0 = 1.0f / sqrtf(a0 / float(p.K) + p.eps);
            inv1 = 1.0f / sqrtf(a1 / float(p.K) + p.eps);
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
                        if (p.epi == BQ_EPI_ADD_RESIDUAL) o += s_res[(ul * 32 + rr) * 16 + m];
                        store_act(p.out, m * p.ldo + n, p.out_dtype, o);
                    }
                }
        }
    }
}

}  // namespace bq
