// Weight-only quantized decode GEMV for sm_100a.
//
//   out[m, n] = epilogue( sum_k xhat[m, k] * W[n, k] ),  xhat = rmsnorm(x) or x
//
// Design (one kernel per linear layer, persistent, 1 CTA per SM):
//  * Work is a 1-D sequence of chunks = (unit, k-block): a unit is 32 output
//    rows (two 16-row MMA tiles; for SiLU*up a 16-row gate tile plus the
//    matching 16-row up tile), a k-block is 128 input features. Chunks are
//    split evenly over all warps of the grid (stream-K): every warp is an
//    independent worker with its own contiguous chunk range.
//  * Each warp streams its weight chunks global->shared through its own ring
//    of TMA tile loads (cp.async.bulk.tensor, mbarrier completion); weights
//    are read exactly once. The first ring fill is issued before the PDL
//    wait, so it overlaps the previous kernel's tail.
//  * The CTA prologue computes the RMSNorm factors (full-K sum of squares)
//    and stages the normalized activations for the CTA's k-range in shared
//    memory, already permuted into m16n8k16 B-fragment order (f16 with a
//    per-row power-of-two scale, or bf16 for bf16 weights).
//  * Weights are dequantized in registers straight into A fragments (int4 via
//    LOP3 + magic-number f16, fp8 via cvt.e4m3x2, int8 via PRMT) and
//    multiplied on the tensor cores: one mma.m16n8k16 covers 16 weight rows
//    x 16 k x 8 activation rows. int4 group scale/zero are applied per group
//    on the fp32 accumulator: sum_k x (q - 8) s + z sum_k x.
//  * A unit split across workers is finished by the last worker to arrive
//    (atomic counter, fixed summation order, no waiting): it sums the
//    partials and runs the epilogue. Counters are reset by that worker.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

__device__ unsigned int g_device_error = 0;

// ------------------------------------------------------------------ traits
template <int FMT>
struct Fmt;
template <>
struct Fmt<BQ_W_BF16> {
    static constexpr int kBoxesPerTile = 4;  // 4 x (16 rows x 32 bf16)
    static constexpr bool kInt4 = false, kF16 = false;
};
template <>
struct Fmt<BQ_W_INT4_TINYGEMM> {
    static constexpr int kBoxesPerTile = 1;  // 2 nTiles x 512 B
    static constexpr bool kInt4 = true, kF16 = true;
    static constexpr int kOfs = 8;
};
template <>
struct Fmt<BQ_W_INT4_PLAIN> {
    static constexpr int kBoxesPerTile = 1;  // 16 rows x 64 B
    static constexpr bool kInt4 = true, kF16 = true;
    static constexpr int kOfs = 0;
};
template <>
struct Fmt<BQ_W_FP8_E4M3> {
    static constexpr int kBoxesPerTile = 2;  // 2 x (16 rows x 64 B)
    static constexpr bool kInt4 = false, kF16 = true;
};
template <>
struct Fmt<BQ_W_INT8> {
    static constexpr int kBoxesPerTile = 2;
    static constexpr bool kInt4 = false, kF16 = true;
};

// Where activation element k (0..127 inside a k-block) sits in the B
// fragments: MMA index i (0..7), register (0: b0, 1: b1), half, lane%4.
struct FragPos {
    int i, reg, half, t;
};
template <int FMT>
__device__ __forceinline__ FragPos frag_pos(int k) {
    FragPos f;
    if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
        // natural m16n8k16 order: k-tile k/16, b0 = {2t, 2t+1}, b1 = {2t+8, 2t+9}
        const int kk = k & 15;
        f.i = k >> 4;
        f.reg = kk >> 3;
        f.half = kk & 1;
        f.t = (kk & 7) >> 1;
    } else if constexpr (FMT == BQ_W_INT4_PLAIN) {
        // lane t holds k = 32t + 8j + s (word j, nibble s)
        const int s = k & 7;
        f.t = k >> 5;
        f.i = 2 * ((k >> 3) & 3) + ((s & 3) >> 1);
        f.reg = s & 1;
        f.half = s >> 2;
    } else if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
        // box h = k/64, lane t holds k = 64h + 16t + 4j + s
        const int r = k & 63, s = r & 3;
        f.t = r >> 4;
        f.i = 4 * (k >> 6) + ((r & 15) >> 2);
        f.reg = s >> 1;
        f.half = s & 1;
    } else {
        // bf16: box h = k/32, lane t holds k = 32h + 8t + 4e + s
        const int r = k & 31, s = r & 3;
        f.t = r >> 3;
        f.i = 2 * (k >> 5) + ((r & 7) >> 2);
        f.reg = s >> 1;
        f.half = s & 1;
    }
    return f;
}

struct SmemLayout {
    uint32_t bars, ring, xfrag, xsum, rowinfo, red, total;
};

__host__ __device__ inline int sz_tile_bytes(int gpk_box) { return ((64 * gpk_box + 127) / 128) * 128; }

__host__ __device__ inline SmemLayout smem_layout(int ring_slots, int slot_bytes, int xfrag_kb, int mt,
                                                  int xsum_groups) {
    SmemLayout L;
    uint32_t o = 0;
    L.bars = o;
    o += kWarpsPerCta * ring_slots * 8;
    o = (o + 1023) & ~1023u;
    L.ring = o;
    o += kWarpsPerCta * ring_slots * slot_bytes;
    L.xfrag = o;
    o += xfrag_kb * mt * 2048;
    L.xsum = o;
    o += xfrag_kb * xsum_groups * 8 * mt * 4;
    L.rowinfo = o;  // inv[16], up-scale[16], down-scale[16]
    o += 3 * 16 * 4;
    L.red = o;  // [8 warps][16]
    o += kWarpsPerCta * 16 * 4;
    L.total = o;
    return L;
}

__device__ __forceinline__ int64_t worker_of(int64_t c, int64_t W, int64_t T) { return ((c + 1) * W - 1) / T; }

// ------------------------------------------------------------------ kernel
template <int FMT, int MT, int GPK>
__global__ void __launch_bounds__(kWarpsPerCta * 32, 1)
    gemv_kernel(const __grid_constant__ CUtensorMap tm_w, const __grid_constant__ CUtensorMap tm_sz,
                const GemvParams p) {
    using F = Fmt<FMT>;
    extern __shared__ __align__(1024) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = lane & 3, tg = lane >> 2;  // lane%4, lane/4
    const int KB = p.kb_count;
    const int64_t T = p.total_chunks, W = p.workers;
    const int gpk_box = FMT == BQ_W_INT4_TINYGEMM ? (p.group >= 128 ? 1 : 128 / p.group) : 1;
    const int szb = F::kInt4 ? sz_tile_bytes(gpk_box) : 0;
    const SmemLayout L = smem_layout(p.ring_slots, p.slot_bytes, p.xfrag_kb, MT, F::kInt4 ? GPK : 0);
    const uint32_t sbase = smem_u32(smem);
    const int RS = p.ring_slots;

    const int64_t wid = int64_t(blockIdx.x) * kWarpsPerCta + warp;
    const bool active = wid < W;
    const int64_t c_begin = active ? wid * T / W : 0;
    const int64_t c_end = active ? (wid + 1) * T / W : 0;
    const int64_t w0 = int64_t(blockIdx.x) * kWarpsPerCta;
    const int64_t w1 = min(w0 + kWarpsPerCta, W);
    const int64_t cta_begin = w0 * T / W, cta_end = w1 * T / W;
    const int kb_first = int(cta_begin % KB);

    const uint32_t my_bars = sbase + L.bars + warp * RS * 8;
    const uint32_t my_ring = sbase + L.ring + warp * RS * p.slot_bytes;
    const uint32_t tx_bytes = 2 * F::kBoxesPerTile * kBoxBytes + (F::kInt4 ? 2 * 64 * gpk_box : 0);

    auto tile_row = [&](int unit, int tile) -> int {
        if (p.epi == BQ_EPI_SILU_MUL) return tile == 0 ? 16 * unit : p.n_half + 16 * unit;
        return 32 * unit + 16 * tile;
    };
    auto issue = [&](int64_t c, int slot) {
        const int unit = int(c / KB), kb = int(c % KB);
        const uint32_t bar = my_bars + slot * 8;
        const uint32_t dst = my_ring + slot * p.slot_bytes;
        mbar_arrive_expect_tx(bar, tx_bytes);
#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
            const int row = tile_row(unit, tile);
#pragma unroll
            for (int b = 0; b < F::kBoxesPerTile; ++b) {
                const uint32_t d = dst + (tile * F::kBoxesPerTile + b) * kBoxBytes;
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
                const int grp = p.group >= 128 ? kb * 128 / p.group : kb * gpk_box;
                tma_load_2d(dst + 2 * F::kBoxesPerTile * kBoxBytes + tile * szb, &tm_sz, 2 * row, grp, bar);
            }
        }
    };

    // ---- barriers + first ring fill (weights are static: before the PDL wait)
    if (lane == 0) {
        for (int s = 0; s < RS; ++s) mbar_init(my_bars + s * 8, 1);
        fence_barrier_init();
        tma_prefetch_desc(&tm_w);
        for (int s = 0; s < RS && c_begin + s < c_end; ++s) issue(c_begin + s, s);
    }
    __syncwarp();
    pdl_launch_dependents();
    pdl_wait();

    // ---- prologue: RMSNorm factors, activation scaling, fragment staging
    float* s_inv = reinterpret_cast<float*>(smem + L.rowinfo);
    float* s_up = s_inv + 16;
    float* s_down = s_inv + 32;
    float* s_red = reinterpret_cast<float*>(smem + L.red);
    const int mrows = 8 * MT;
    const int M = p.M;
    const bool norm = p.gamma != nullptr;
    const __nv_bfloat16* gamma = static_cast<const __nv_bfloat16*>(p.gamma);
    const int nkb = p.xfrag_kb;

    if (norm) {
        for (int m = 0; m < M; ++m) {
            float ss = 0.f;
            for (int k = threadIdx.x; k < p.K; k += blockDim.x) {
                const float v = load_act(p.x, m * p.ldx + k, p.x_dtype);
                ss = fmaf(v, v, ss);
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0) s_red[warp * 16 + m] = ss;
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            float ss = 0.f;
            if (threadIdx.x < M)
                for (int w = 0; w < kWarpsPerCta; ++w) ss += s_red[w * 16 + threadIdx.x];
            s_inv[threadIdx.x] = 1.0f / sqrtf(ss / float(p.K) + p.eps);
        }
        __syncthreads();
    } else if (threadIdx.x < 16) {
        s_inv[threadIdx.x] = 1.0f;
    }
    // per-row power-of-two scale so the f16 activations use the full range
    if constexpr (F::kF16) {
        for (int m = 0; m < M; ++m) {
            float amax = 0.f;
            for (int e = threadIdx.x; e < nkb * kKB; e += blockDim.x) {
                const int kb = (kb_first + e / kKB) % KB;
                const int k = kb * kKB + (e % kKB);
                float v = load_act(p.x, m * p.ldx + k, p.x_dtype);
                if (norm) v *= __bfloat162float(gamma[k]);
                amax = fmaxf(amax, fabsf(v));
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
            if (lane == 0) s_red[warp * 16 + m] = amax;
        }
        __syncthreads();
        if (threadIdx.x < 16) {
            float amax = 0.f;
            if (threadIdx.x < M)
                for (int w = 0; w < kWarpsPerCta; ++w) amax = fmaxf(amax, s_red[w * 16 + threadIdx.x]);
            amax *= s_inv[threadIdx.x];
            int e = 0;
            if (amax > 0.f && amax < INFINITY) {
                int ex;
                frexpf(amax, &ex);
                e = min(max(ex - 15, -100), 100);  // amax * 2^-e in [2^14, 2^15)
            }
            s_up[threadIdx.x] = ldexpf(1.0f, e);
            s_down[threadIdx.x] = ldexpf(1.0f, -e);
        }
    } else if (threadIdx.x < 16) {
        s_up[threadIdx.x] = 1.0f;
        s_down[threadIdx.x] = 1.0f;
    }
    __syncthreads();
    {
        uint16_t* xf = reinterpret_cast<uint16_t*>(smem + L.xfrag);
        float* xs = reinterpret_cast<float*>(smem + L.xsum);
        const int vecs = mrows * nkb * 16;  // 8-element vectors, multiple of 128
        const int gsub = F::kInt4 ? (p.group < 128 ? p.group : 128) : 128;
        const int vpg = gsub / 8;  // vectors per group sum: 4, 8 or 16
        for (int f = threadIdx.x; f < vecs; f += blockDim.x) {
            const int v = f & 15;
            const int l = (f >> 4) % nkb;
            const int m = (f >> 4) / nkb;
            const int kb = (kb_first + l) % KB;
            const int mt = m >> 3;
            float vals[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int k = kb * kKB + v * 8 + e;
                float xv = 0.f;
                if (m < M) {
                    xv = load_act(p.x, m * p.ldx + k, p.x_dtype) * s_inv[m];
                    if (norm) xv *= __bfloat162float(gamma[k]);
                    xv *= s_down[m];
                }
                vals[e] = xv;
            }
            float gsum = 0.f;
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const int kin = v * 8 + e;
                const FragPos fp = frag_pos<FMT>(kin);
                uint16_t hbits;
                float rounded;
                if constexpr (F::kF16) {
                    const __half h = __float2half_rn(vals[e]);
                    hbits = __half_as_ushort(h);
                    rounded = __half2float(h);
                } else {
                    const __nv_bfloat16 h = __float2bfloat16_rn(vals[e]);
                    hbits = __bfloat16_as_ushort(h);
                    rounded = __bfloat162float(h);
                }
                gsum += rounded;
                const int ln = 4 * (m & 7) + fp.t;
                const int idx = (((l * MT + mt) * 4 + (fp.i >> 1)) * 32 + ln) * 8 + ((fp.i & 1) * 2 + fp.reg) * 2 + fp.half;
                xf[idx] = hbits;
            }
            if constexpr (F::kInt4) {
                for (int o = 1; o < vpg; o <<= 1) gsum += __shfl_xor_sync(0xffffffffu, gsum, o);
                if ((v % vpg) == 0) {
                    const int sg = v / vpg;  // sub-group inside the k-block
                    xs[((l * GPK + sg) * mrows) + m] = gsum;
                }
            }
        }
    }
    __syncthreads();
    if (!active) return;

    // ---- main loop
    float acc[2][MT][4];
#pragma unroll
    for (int a = 0; a < 2; ++a)
#pragma unroll
        for (int b = 0; b < MT; ++b)
#pragma unroll
            for (int c = 0; c < 4; ++c) acc[a][b][c] = 0.f;

    int cur_unit = -1, seg_first = 0, seg_last = 0;
    const uint32_t xf_base = sbase + L.xfrag;
    const uint32_t xs_base = sbase + L.xsum;

    // flush: finish the current unit segment (direct epilogue or stream-K fixup)
    auto flush = [&](int unit) {
        // back to true scale: column m of the C fragment is 8*mt + 2*tq + (j&1)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const float u0 = s_up[8 * mt + 2 * tq], u1 = s_up[8 * mt + 2 * tq + 1];
#pragma unroll
            for (int tile = 0; tile < 2; ++tile) {
                acc[tile][mt][0] *= u0;
                acc[tile][mt][1] *= u1;
                acc[tile][mt][2] *= u0;
                acc[tile][mt][3] *= u1;
            }
        }
        const bool full = seg_first == 0 && seg_last == KB - 1;
        if (!full) {
            const int64_t wf = worker_of(int64_t(unit) * KB, W, T);
            const int64_t wl = worker_of(int64_t(unit + 1) * KB - 1, W, T);
            const int npieces = int(wl - wf + 1);
            const int me = int(wid - wf);
            float* base = p.partials + (int64_t(unit) * p.p_max) * (2 * MT * 128);
            float* mine = base + int64_t(me) * (2 * MT * 128);
#pragma unroll
            for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
                    __stcg(reinterpret_cast<float4*>(mine + ((tile * MT + mt) * 32 + lane) * 4),
                           make_float4(acc[tile][mt][0], acc[tile][mt][1], acc[tile][mt][2], acc[tile][mt][3]));
            __threadfence();
            __syncwarp();
            unsigned int old = 0;
            if (lane == 0) old = atomicAdd(p.counters + unit, 1u);
            old = __shfl_sync(0xffffffffu, old, 0);
            if (old != unsigned(npieces - 1)) return;  // not last: done with this unit
            __threadfence();
            float tot[2][MT][4];
#pragma unroll
            for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) tot[tile][mt][j] = 0.f;
            for (int q = 0; q < npieces; ++q) {
#pragma unroll
                for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        float4 v;
                        if (q == me)
                            v = make_float4(acc[tile][mt][0], acc[tile][mt][1], acc[tile][mt][2], acc[tile][mt][3]);
                        else
                            v = ldcg_f4(base + int64_t(q) * (2 * MT * 128) + ((tile * MT + mt) * 32 + lane) * 4);
                        tot[tile][mt][0] += v.x;
                        tot[tile][mt][1] += v.y;
                        tot[tile][mt][2] += v.z;
                        tot[tile][mt][3] += v.w;
                    }
            }
            if (lane == 0) atomicExch(p.counters + unit, 0u);
#pragma unroll
            for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[tile][mt][j] = tot[tile][mt][j];
        }
        // ---- epilogue on the finished unit
        const float* wscale = static_cast<const float*>(p.scale);
#pragma unroll
        for (int tile = 0; tile < 2; ++tile)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = tile_row(unit, tile) + tg + (j >> 1) * 8;
                float sc = 1.0f, bi = 0.0f;
                if (n < p.N) {
                    if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                        sc = wscale[n];
                        if (FMT == BQ_W_INT8 && (p.flags & BQ_FLAG_SCALE_ROUND_BF16))
                            sc = __bfloat162float(__float2bfloat16_rn(sc));
                    }
                    if (p.bias) bi = load_act(p.bias, n, p.out_dtype);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) acc[tile][mt][j] = acc[tile][mt][j] * sc + bi;
            }
        if (p.epi == BQ_EPI_SILU_MUL) {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int n = 16 * unit + tg + (j >> 1) * 8;
                    const int m = 8 * mt + 2 * tq + (j & 1);
                    if (n < p.n_half && m < M)
                        store_act(p.out, m * p.ldo + n, p.out_dtype, silu(acc[0][mt][j]) * acc[1][mt][j]);
                }
        } else {
#pragma unroll
            for (int tile = 0; tile < 2; ++tile)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                    for (int j = 0; j < 4; ++j) {
                        const int n = tile_row(unit, tile) + tg + (j >> 1) * 8;
                        const int m = 8 * mt + 2 * tq + (j & 1);
                        if (n < p.N && m < M) {
                            float v = acc[tile][mt][j];
                            if (p.epi == BQ_EPI_ADD_RESIDUAL) v += load_act(p.residual, m * p.ldr + n, p.res_dtype);
                            store_act(p.out, m * p.ldo + n, p.out_dtype, v);
                        }
                    }
        }
    };

    int it = 0;
    for (int64_t c = c_begin; c < c_end; ++c, ++it) {
        const int slot = it % RS;
        const uint32_t parity = (it / RS) & 1;
        if (!mbar_wait(my_bars + slot * 8, parity)) {
            // give up: let the copies still in flight land before exiting
            for (int q = 1; q < RS && c + q < c_end; ++q)
                mbar_wait(my_bars + ((it + q) % RS) * 8, ((it + q) / RS) & 1);
            return;
        }
        const int unit = int(c / KB), kb = int(c % KB);
        if (unit != cur_unit) {
            if (cur_unit >= 0) flush(cur_unit);
            cur_unit = unit;
            seg_first = kb;
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int b = 0; b < MT; ++b)
#pragma unroll
                    for (int j = 0; j < 4; ++j) acc[a][b][j] = 0.f;
        }
        seg_last = kb;
        const int l = (kb - kb_first + KB) % KB;
        const uint32_t src = my_ring + slot * p.slot_bytes;

        // activation fragments for this k-block
        uint32_t bfr[MT][16];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint4 v = lds128(xf_base + (((l * MT + mt) * 4 + q) * 32 + lane) * 16);
                bfr[mt][4 * q + 0] = v.x;
                bfr[mt][4 * q + 1] = v.y;
                bfr[mt][4 * q + 2] = v.z;
                bfr[mt][4 * q + 3] = v.w;
            }

#pragma unroll
        for (int tile = 0; tile < 2; ++tile) {
            if constexpr (F::kInt4) {
                const uint4 r0 = lds128(src + tile * kBoxBytes + lane * 16);
                const uint4 r1 = lds128(src + tile * kBoxBytes + 512 + lane * 16);
                const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                const uint32_t szs = src + 2 * kBoxBytes + tile * szb;
#pragma unroll
                for (int sg = 0; sg < GPK; ++sg) {
                    float c[MT][4];
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int j = 0; j < 4; ++j) c[mt][j] = 0.f;
#pragma unroll
                    for (int ii = 0; ii < 8 / GPK; ++ii) {
                        const int i = sg * (8 / GPK) + ii;
                        const uint32_t x0 = (i & 1) ? (w0[i >> 1] >> 8) : w0[i >> 1];
                        const uint32_t x1 = (i & 1) ? (w1[i >> 1] >> 8) : w1[i >> 1];
                        const uint32_t a0 = i4lo_to_f16x2<F::kOfs>(x0);
                        const uint32_t a2 = i4hi_to_f16x2<F::kOfs>(x0);
                        const uint32_t a1 = i4lo_to_f16x2<F::kOfs>(x1);
                        const uint32_t a3 = i4hi_to_f16x2<F::kOfs>(x1);
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) mma_f16(c[mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                    }
                    const int gi = (p.group >= 128) ? 0 : sg;
                    const uint32_t sz0 = lds32(szs + gi * 64 + tg * 4);
                    const uint32_t sz1 = lds32(szs + gi * 64 + (tg + 8) * 4);
                    const float s0 = __uint_as_float(sz0 << 16), z0 = __uint_as_float(sz0 & 0xFFFF0000u);
                    const float s1 = __uint_as_float(sz1 << 16), z1 = __uint_as_float(sz1 & 0xFFFF0000u);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        const float2 X = lds_f2(xs_base + (((l * GPK + sg) * mrows) + 8 * mt + 2 * tq) * 4);
                        acc[tile][mt][0] += s0 * c[mt][0] + z0 * X.x;
                        acc[tile][mt][1] += s0 * c[mt][1] + z0 * X.y;
                        acc[tile][mt][2] += s1 * c[mt][2] + z1 * X.x;
                        acc[tile][mt][3] += s1 * c[mt][3] + z1 * X.y;
                    }
                }
            } else {
#pragma unroll
                for (int b = 0; b < F::kBoxesPerTile; ++b) {
                    const uint32_t box = src + (tile * F::kBoxesPerTile + b) * kBoxBytes;
                    const uint4 r0 = lds128(box + lane * 16);
                    const uint4 r1 = lds128(box + 512 + lane * 16);
                    const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                    const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                    if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                        for (int e = 0; e < 2; ++e) {
                            const int i = 2 * b + e;
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_bf16(acc[tile][mt], w0[2 * e], w1[2 * e], w0[2 * e + 1], w1[2 * e + 1],
                                         bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 4; ++j) {
                            const int i = 4 * b + j;
                            uint32_t a0, a1, a2, a3;
                            if constexpr (FMT == BQ_W_FP8_E4M3) {
                                a0 = e4m3x2_to_f16x2(uint16_t(w0[j] & 0xFFFF));
                                a2 = e4m3x2_to_f16x2(uint16_t(w0[j] >> 16));
                                a1 = e4m3x2_to_f16x2(uint16_t(w1[j] & 0xFFFF));
                                a3 = e4m3x2_to_f16x2(uint16_t(w1[j] >> 16));
                            } else {
                                const uint32_t x0 = w0[j] ^ 0x80808080u, x1 = w1[j] ^ 0x80808080u;
                                a0 = i8pair_to_f16x2(x0, 0x4140u);
                                a2 = i8pair_to_f16x2(x0, 0x4342u);
                                a1 = i8pair_to_f16x2(x1, 0x4140u);
                                a3 = i8pair_to_f16x2(x1, 0x4342u);
                            }
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_f16(acc[tile][mt], a0, a1, a2, a3, bfr[mt][2 * i], bfr[mt][2 * i + 1]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0 && c + RS < c_end) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            issue(c + RS, slot);
        }
    }
    if (cur_unit >= 0) flush(cur_unit);
}

// ------------------------------------------------------------------ host side
namespace {

struct KernelEntry {
    const void* fn;
};

template <int FMT, int MT, int GPK>
const void* kernel_ptr() {
    return reinterpret_cast<const void*>(&gemv_kernel<FMT, MT, GPK>);
}

const void* pick_kernel(int fmt, int mt, int gpk) {
#define BQ_K(F)                                                          \
    if (fmt == F) {                                                      \
        if (mt == 1) return gpk == 1 ? kernel_ptr<F, 1, 1>() : nullptr;  \
        return gpk == 1 ? kernel_ptr<F, 2, 1>() : nullptr;               \
    }
    BQ_K(BQ_W_BF16)
    BQ_K(BQ_W_INT4_PLAIN)
    BQ_K(BQ_W_FP8_E4M3)
    BQ_K(BQ_W_INT8)
#undef BQ_K
    if (fmt == BQ_W_INT4_TINYGEMM) {
        if (mt == 1) {
            if (gpk == 1) return kernel_ptr<BQ_W_INT4_TINYGEMM, 1, 1>();
            if (gpk == 2) return kernel_ptr<BQ_W_INT4_TINYGEMM, 1, 2>();
            if (gpk == 4) return kernel_ptr<BQ_W_INT4_TINYGEMM, 1, 4>();
        } else {
            if (gpk == 1) return kernel_ptr<BQ_W_INT4_TINYGEMM, 2, 1>();
            if (gpk == 2) return kernel_ptr<BQ_W_INT4_TINYGEMM, 2, 2>();
            if (gpk == 4) return kernel_ptr<BQ_W_INT4_TINYGEMM, 2, 4>();
        }
    }
    return nullptr;
}

int boxes_per_tile(int fmt) {
    switch (fmt) {
        case BQ_W_BF16: return 4;
        case BQ_W_FP8_E4M3:
        case BQ_W_INT8: return 2;
        default: return 1;
    }
}

bool is_int4(int fmt) { return fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN; }

}  // namespace

// Shape plan shared by the workspace query and the launch.
int plan_gemv(const bq_gemv_desc* d, int rows, GemvPlan* pl) {
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    pl->mt = rows > 8 ? 2 : 1;
    const int fmt = d->wfmt;
    pl->gpk = 1;
    if (fmt == BQ_W_INT4_TINYGEMM) pl->gpk = d->group >= 128 ? 1 : 128 / d->group;
    const int kb = d->K / kKB;
    const int64_t n_units = d->epilogue == BQ_EPI_SILU_MUL ? (d->N / 2 + 15) / 16 : (d->N + 31) / 32;
    const int64_t T = n_units * kb;
    if (n_units > kMaxUnits)
        return set_error(BQ_ERR_SHAPE, "N=%d too large (at most %d 32-row units)", d->N, kMaxUnits);
    const int gpk_box = pl->gpk;
    const int slot = 2 * boxes_per_tile(fmt) * kBoxBytes + (is_int4(fmt) ? 2 * sz_tile_bytes(gpk_box) : 0);
    pl->slot_bytes = slot;
    int grid = dev->sm_count;
    int ring = std::max(2, std::min(8, (12 * 1024) / slot));
    for (int attempt = 0; attempt < 16; ++attempt) {
        const int64_t maxW = int64_t(grid) * kWarpsPerCta;
        const int64_t W = std::min<int64_t>(maxW, T);
        const int g = int((W + kWarpsPerCta - 1) / kWarpsPerCta);
        const int64_t per_worker = (T + W - 1) / W;
        const int xkb = int(std::min<int64_t>(kb, per_worker * kWarpsPerCta + 1));
        const SmemLayout L = smem_layout(ring, slot, xkb, pl->mt, is_int4(fmt) ? pl->gpk : 0);
        if (L.total <= uint32_t(dev->smem_optin)) {
            const int64_t cmin = T / W;
            int64_t pmax = std::min<int64_t>(kb, (kb - 1 + cmin - 1) / cmin + 1);
            pl->grid = g;
            pl->workers = int(W);
            pl->ring_slots = ring;
            pl->xfrag_kb = xkb;
            pl->smem = L.total;
            pl->n_units = int(n_units);
            pl->total_chunks = T;
            pl->p_max = int(std::max<int64_t>(pmax, 1));
            pl->counters_bytes = kCounterBytes;
            pl->partials_bytes = n_units * int64_t(pl->p_max) * 2 * pl->mt * 128 * 4;
            return BQ_OK;
        }
        if (ring > 2)
            --ring;
        else
            grid *= 2;
    }
    return set_error(BQ_ERR_SHAPE, "GEMV shape does not fit in shared memory (K=%d, M tile %d)", d->K, pl->mt);
}

int launch_gemv(const bq_gemv_desc* d, const GemvPlan& pl, int row0, int rows, void* workspace,
                cudaStream_t stream) {
    const int fmt = d->wfmt;
    const void* fn = pick_kernel(fmt, pl.mt, pl.gpk);
    if (!fn) return set_error(BQ_ERR_FORMAT, "no kernel for format %d (group %d)", fmt, d->group);
    CUtensorMap tm_w, tm_sz;
    int rc = encode_weight_maps(d, &tm_w, &tm_sz);
    if (rc) return rc;

    GemvParams p;
    std::memset(&p, 0, sizeof(p));
    p.M = rows;
    p.N = d->N;
    p.K = d->K;
    p.n_units = pl.n_units;
    p.kb_count = d->K / kKB;
    p.epi = d->epilogue;
    p.group = d->group;
    p.x_dtype = d->x_dtype;
    p.out_dtype = d->out_dtype;
    p.res_dtype = d->res_dtype;
    p.flags = d->flags;
    p.eps = d->eps;
    p.n_half = d->N / 2;
    p.workers = pl.workers;
    p.total_chunks = pl.total_chunks;
    p.p_max = pl.p_max;
    p.ring_slots = pl.ring_slots;
    p.slot_bytes = pl.slot_bytes;
    p.xfrag_kb = pl.xfrag_kb;
    const int xs = dtype_size(d->x_dtype), os = dtype_size(d->out_dtype), rs = dtype_size(d->res_dtype);
    p.x = static_cast<const char*>(d->x) + int64_t(row0) * d->ldx * xs;
    p.ldx = d->ldx;
    p.gamma = d->gamma;
    p.scale = d->scale;
    p.bias = d->bias;
    p.residual = d->residual ? static_cast<const char*>(d->residual) + int64_t(row0) * d->ldr * rs : nullptr;
    p.ldr = d->ldr;
    p.out = static_cast<char*>(d->out) + int64_t(row0) * d->ldo * os;
    p.ldo = d->ldo;
    p.counters = static_cast<unsigned int*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + pl.counters_bytes);

    rc = ensure_smem_attr(fn, pl.smem);
    if (rc) return rc;

    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kWarpsPerCta * 32);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    if (d->flags & BQ_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    void* args[] = {&tm_w, &tm_sz, &p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "GEMV launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // namespace bq
