// Tensor-core GEMV for 17..128 activation rows: every weight byte is read once
// whatever the row count (the mma.sync kernel re-streams the weights once per
// 16 rows). Same contract as bq_gemv (models/fused/kernels.py:334-351,
// models/int4_linear.py:99-109 -- tinygemm's single pass over the weights at
// any M --, models/fp8_linear.py:68-83, models/int8_linear.py:50-53).
//
// One CTA per SM, 14 warps:
//   warps 0-7  dequantizers, two groups of four. Group g takes the CTA's
//              k-blocks g, g+2, ...; thread r of a group owns weight row r of
//              the 128-row unit. It streams its own row's bytes with cp.async
//              into a private ring (no cross-thread hand-off of raw data),
//              dequantizes 128 k at a time to bf16 in registers and writes
//              them with tcgen05.st into its tensor-memory (TMEM) lane: the
//              MMA's A operand lives in TMEM, so dequantized weights never
//              touch shared memory.
//   warp 8     activation loader: cp.async of the k-block's X tile (bf16
//              rows, K-major core matrices) into one of four shared-memory
//              stages; each lane's copies complete on the stage's mbarrier
//              (cp.async.mbarrier.arrive.noinc), so the loader runs up to
//              four k-blocks ahead of the tensor cores.
//   warp 9     allocates TMEM; one thread issues tcgen05.mma kind::f16
//              (M = 128 weight rows, N = rows rounded up to 16, K = 16; A from
//              TMEM, B from shared memory, fp32 accumulators in TMEM) and
//              tcgen05.commit to free stages / publish the accumulator.
//   warps 10-13 copy the accumulator (tcgen05.ld, one TMEM lane quadrant per
//              warp) into shared memory once the last MMA is done.
//
// Work split: a unit is 128 weight rows (SiLU*up: 64 gate rows and the
// matching 64 up rows). The C CTAs of unit u form a thread-block cluster;
// cluster rank r takes the k-blocks [r KB / C, (r + 1) KB / C). C is chosen so
// that units x C fills the SMs in one wave (O and down projections: 16 units
// x 8 slices; gate+up: 128 units x 1). After a cluster barrier every CTA sums
// its share of the unit's rows over the C partial accumulators in rank order
// (distributed shared memory; deterministic), applies the per-row scale,
// bias, SiLU*up or residual, and stores; a second barrier keeps each CTA's
// shared memory alive until the others have read it. No global scratch and
// no cross-CTA counters.
//
// With an RMSNorm the rows are normalized first by a short kernel into the
// workspace (bf16 x * rstd * gamma, as models/fused/kernels.py:541
// rmsnorm_kernel computes it); programmatic dependent launch lets the weight
// stream of the GEMV start while it runs.
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <array>
#include <cstring>
#include <map>
#include <mutex>
#include <utility>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {
namespace {

constexpr int kTcWarps = 15;
constexpr int kTcThreads = kTcWarps * 32;
constexpr int kTcXWarp = 8;
constexpr int kTcMmaWarp = 9;
constexpr int kTcStages = 4;       // A (TMEM) and X (shared) stages, indexed by block % 4
constexpr int kTcTmemCols = 512;
constexpr int kTcACol0 = 256;      // A stage a at columns 256 + 64 a (accumulator at columns 0..N-1)
constexpr int kTcACols = 64;       // 128 bf16 k-values of one row = 64 32-bit columns
constexpr int kTcProdWarp = 14;   // weight producer (TMA)
constexpr int kTcMaxWStages = 8;   // weight ring stages at most
constexpr int kTcMinRows = 17;
constexpr int kTcMaxRows = 128;

struct TcParams {
    CUtensorMap xmap;  // activation rows [M][K] bf16, boxes of 64 k x n_mma rows, 128-byte swizzle
    CUtensorMap wmap;  // weights: int4 plain / 8-bit / bf16 2-D, tinygemm 3-D (see tc_encode_weights)
    const void* w;
    const void* scale;
    const void* bias;
    const void* residual;
    void* out;
    const __nv_bfloat16* x;
    long long ldx, ldr, ldo;
    int M, N, K, KB, group, epi, out_dtype, res_dtype;
    unsigned flags;
    int C, n_mma, wst;  // cluster size, MMA N, weight ring stages
    unsigned idesc;
    long long wait_cycles;
    unsigned sm_x, sm_w, sm_bar, sm_total, red_pitch;
    unsigned w_stage;   // bytes per weight stage: 128 rows of weights, then int4 scales
    unsigned w_bytes;   // weight bytes per stage (the scales follow)
    unsigned tx_bytes;  // bytes a stage receives per k-block (weights + scales)
};

// Bytes of one weight row per 128-k block, by format.
__host__ __device__ constexpr int tc_row_bytes(int fmt) {
    return (fmt == BQ_W_INT4_TINYGEMM || fmt == BQ_W_INT4_PLAIN) ? 64 : fmt == BQ_W_BF16 ? 256 : 128;
}

// ------------------------------------------------------------- tcgen05 / TMEM
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(cols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16};" ::"r"(taddr),
        "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]), "r"(v[8]), "r"(v[9]),
        "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
        : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// D[tmem] (+)= A[tmem] . B[smem]^T, one 128 x N x 16 step.
__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The mbarrier completes one phase once every tcgen05 op issued so far by this thread is done.
__device__ __forceinline__ void tc_commit(uint32_t bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
                 : "memory");
}

// Shared-memory matrix descriptor of the K-major bf16 activation tile as the
// tensor map writes it: rows of 64 k (128 B) in 128-byte swizzle atoms of 8
// rows; a k16 step inside the atom starts 32 B further (the swizzle is applied
// to the final address); bit 46 is the sm_100 descriptor version.
__device__ __forceinline__ uint64_t tc_bdesc(uint32_t saddr) {
    // K-major, 128-byte swizzle: 8-row groups 1024 B apart (stride offset); the
    // leading offset is unused for swizzled K-major layouts; layout type 2 = 128B
    return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) | (1ull << 46) |
           (uint64_t(2) << 61);
}

// Tiled TMA load of a 2-D box (no multicast), completion on an mbarrier.
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar)
                 : "memory");
}

// ------------------------------------------------------------- small helpers
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// Barrier of the 128 epilogue threads that also returns whether any of them passed `pred`.
__device__ __forceinline__ bool epi_any(bool pred) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 p, %1, 0;\n\t"
        "bar.red.or.pred q, 1, 128, p;\n\t"
        "selp.u32 %0, 1, 0, q;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(pred))
        : "memory");
    return r != 0;
}

// f16 pair -> bf16 pair (exact for the e4m3 values it is used on).
__device__ __forceinline__ uint32_t f16x2_to_bf16x2(uint32_t h) {
    __half2 hh;
    memcpy(&hh, &h, 4);
    const float2 f = __half22float2(hh);
    return pack_bf162(f.x, f.y);
}

constexpr uint32_t kOne2 = 0x3F803F80u;   // bf16 (1, 1)
constexpr uint32_t kM136x2 = 0xC308C308u; // bf16 (-136, -136)
constexpr uint32_t kM128x2 = 0xC300C300u; // bf16 (-128, -128)

// Waits for a phase of `bar` with a bound; gives up when another role has
// already given up (abort flag) or after p.wait_cycles, recording the timeout.
__device__ __forceinline__ bool tc_wait(uint32_t bar, uint32_t parity, volatile int* abort, long long limit) {
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    for (int it = 0;; ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 15) == 15) {
            if (abort && *abort) return false;
            if (clock64() - t0 > limit) {
                atomicOr(&g_device_error, BQ_DEVERR_WAIT_TIMEOUT_BIT);
                if (abort) *abort = 1;
                return false;
            }
        }
    }
}

// Weight row of lane r of unit u.
__device__ __forceinline__ int tc_row(const TcParams& p, int u, int r) {
    if (p.epi == BQ_EPI_SILU_MUL) return r < 64 ? u * 64 + r : (p.N >> 1) + u * 64 + (r - 64);
    return u * 128 + r;
}

// ------------------------------------------------------------- weight stream
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, uint32_t bar) {
    asm volatile("cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];"
                 ::"r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
                 : "memory");
}
// 1-D bulk copy global -> shared (16-byte aligned, size a multiple of 16).
__device__ __forceinline__ void tc_bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// One k-block of unit u into weight stage `st` (one thread): the 128 rows (two
// 64-row boxes for SiLU*up: gate rows, then the matching up rows), then for
// int4 the (scale, zero) words of the block's groups, [group][128 rows].
template <int FMT>
__device__ __forceinline__ void tc_produce(const TcParams& p, int u, int kb, uint32_t st, uint32_t bar) {
    const bool silu = p.epi == BQ_EPI_SILU_MUL;
    const int nbox = silu ? 2 : 1, brows = silu ? 64 : 128;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        if (h >= nbox) break;
        const int row0 = silu ? (h == 0 ? u * 64 : (p.N >> 1) + u * 64) : u * 128;
        constexpr int line = FMT == BQ_W_BF16 ? 128 : tc_row_bytes(FMT);  // bytes of a row in one box
        const uint32_t dst = st + uint32_t(h * brows * line);
        if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
            tma_load_3d(dst, &p.wmap, 0, kb, row0 >> 3, bar);  // [n8][512 B]: the 8-row tiles of k-block kb
        } else if constexpr (FMT == BQ_W_INT4_PLAIN) {
            tma_load_2d(dst, &p.wmap, kb * 64, row0, bar);
        } else if constexpr (FMT == BQ_W_BF16) {
            tma_load_2d(dst, &p.wmap, kb * 128, row0, bar);                      // k 0-63 of the block
            tma_load_2d(dst + 128u * 128u, &p.wmap, kb * 128 + 64, row0, bar);   // k 64-127
        } else {
            tma_load_2d(dst, &p.wmap, kb * 128, row0, bar);
        }
    }
    if constexpr (FMT == BQ_W_INT4_TINYGEMM || FMT == BQ_W_INT4_PLAIN) {
        const int g = p.group;
        const int ngr = g < 128 ? 128 / g : 1;
        const int g0 = g <= 128 ? kb * (128 / g) : kb / (g / 128);
        const char* s = static_cast<const char*>(p.scale);
        for (int gi = 0; gi < ngr; ++gi) {
            const uint32_t dsc = st + p.w_bytes + uint32_t(gi * 512);
            if (silu) {
                tc_bulk_g2s(dsc, s + (size_t(g0 + gi) * p.N + u * 64) * 4, 256, bar);
                tc_bulk_g2s(dsc + 256, s + (size_t(g0 + gi) * p.N + (p.N >> 1) + u * 64) * 4, 256, bar);
            } else {
                tc_bulk_g2s(dsc, s + (size_t(g0 + gi) * p.N + u * 128) * 4, 512, bar);
            }
        }
    }
}

// 16-byte chunk c of weight row r in a stage, as the tensor map's swizzle placed
// it: int4 rows are 64 B (64-byte swizzle: chunk ^ bits 1-2 of the row), 8-bit
// rows 128 B (128-byte swizzle: chunk ^ row % 8), bf16 two 128-byte halves.
template <int FMT>
__device__ __forceinline__ uint32_t tc_chunk(uint32_t st, int r, int c) {
    if constexpr (FMT == BQ_W_INT4_TINYGEMM)
        return st + uint32_t(r * 64 + 16 * c);  // 512-byte tiles copied as they are stored (no swizzle)
    else if constexpr (FMT == BQ_W_INT4_PLAIN)
        return st + uint32_t(r * 64 + 16 * (c ^ ((r >> 1) & 3)));
    else if constexpr (FMT == BQ_W_BF16)
        return st + uint32_t((c >> 3) * 128 * 128 + r * 128 + 16 * ((c & 7) ^ (r & 7)));
    else
        return st + uint32_t(r * 128 + 16 * (c ^ (r & 7)));
}

// Dequantizes row r's block from weight stage `st` into bf16 pairs (low half =
// even k) and stores them to TMEM columns col .. col+63 of the warp's lane.
template <int FMT>
__device__ __forceinline__ void tc_dequant(const TcParams& p, int r, uint32_t st, uint32_t taddr) {
    const uint32_t sc = st + p.w_bytes;
    if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
        // word j of lane c, nibble pair i (bits 4i and 16 + 4i) holds the codes of
        // k = 32 j + 8 i + 2 c and k + 1 (even k in the low nibble of the pair)
        uint4 l[4];
#pragma unroll
        for (int c = 0; c < 4; ++c) l[c] = lds128(tc_chunk<FMT>(st, r, c));
        const int g = p.group;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int gi = g == 32 ? j : g == 64 ? (j >> 1) : 0;
            const uint32_t sz = lds32(sc + gi * 512 + r * 4);
            const uint32_t s2 = prmt(sz, sz, 0x1010u), z2 = prmt(sz, sz, 0x3232u);
            uint32_t o[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint32_t wj = j == 0 ? l[c].x : j == 1 ? l[c].y : j == 2 ? l[c].z : l[c].w;
#pragma unroll
                for (int i = 0; i < 4; ++i) {
                    const uint32_t q = bf16x2_fma(i4_bf16(wj >> (4 * i)), kOne2, kM136x2);  // q - 8, exact
                    o[4 * i + c] = bf16x2_fma(q, s2, z2);  // (q - 8) * scale + zero, one rounding
                }
            }
            tmem_st16(taddr + 16 * j, o);
        }
    } else if constexpr (FMT == BQ_W_INT4_PLAIN) {
        // byte b of the row holds k = 2b (low nibble) and 2b + 1 (high nibble)
        const uint32_t sz = lds32(sc + r * 4);
        const uint32_t s2 = prmt(sz, sz, 0x1010u), m2 = prmt(sz, sz, 0x3232u);
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            const uint4 l = lds128(tc_chunk<FMT>(st, r, c));
            uint32_t o[16];
#pragma unroll
            for (int t = 0; t < 4; ++t) {
                const uint32_t wt = t == 0 ? l.x : t == 1 ? l.y : t == 2 ? l.z : l.w;
                const uint32_t lo = wt & 0x0F0F0F0Fu, hi = (wt >> 4) & 0x0F0F0F0Fu;
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    // bytes (lo.b, 0, hi.b, 0): a selector nibble with bit 3 set copies the sign of a byte < 16
                    const uint32_t sel = b | ((8 | b) << 4) | ((4 + b) << 8) | ((12 + b) << 12);
                    const uint32_t q = bf16x2_fma(prmt(lo, hi, sel) | 0x43004300u, kOne2, kM128x2);  // q, exact
                    o[4 * t + b] = bf16x2_fma(q, s2, m2);  // q * scale + min, one rounding
                }
            }
            tmem_st16(taddr + 16 * c, o);
        }
    } else if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t o[16];
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const uint4 l = lds128(tc_chunk<FMT>(st, r, 4 * j + c));
                o[4 * c] = l.x;
                o[4 * c + 1] = l.y;
                o[4 * c + 2] = l.z;
                o[4 * c + 3] = l.w;
            }
            tmem_st16(taddr + 16 * j, o);
        }
    } else {
        // fp8 / int8: chunk c holds k = 16 c .. 16 c + 15; bf16 represents both exactly
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            uint32_t o[16];
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const uint4 l = lds128(tc_chunk<FMT>(st, r, 2 * j + h));
#pragma unroll
                for (int t = 0; t < 4; ++t) {
                    const uint32_t wt = t == 0 ? l.x : t == 1 ? l.y : t == 2 ? l.z : l.w;
                    if constexpr (FMT == BQ_W_FP8_E4M3) {
                        o[8 * h + 2 * t] = f16x2_to_bf16x2(e4m3x2_to_f16x2(uint16_t(wt & 0xFFFFu)));
                        o[8 * h + 2 * t + 1] = f16x2_to_bf16x2(e4m3x2_to_f16x2(uint16_t(wt >> 16)));
                    } else {
                        const int v = int(wt);
                        o[8 * h + 2 * t] = pack_bf162(float((v << 24) >> 24), float((v << 16) >> 24));
                        o[8 * h + 2 * t + 1] = pack_bf162(float((v << 8) >> 24), float(v >> 24));
                    }
                }
            }
            tmem_st16(taddr + 16 * j, o);
        }
    }
}

// Output of activation row m for weight row n (unit-relative row r), value v.
__device__ __forceinline__ void tc_store(const TcParams& p, int m, int n, float v) {
    if (p.epi == BQ_EPI_ADD_RESIDUAL) v += load_act(p.residual, m * p.ldr + n, p.res_dtype);
    store_act(p.out, m * p.ldo + n, p.out_dtype, v);
}

template <int FMT>
__global__ void __launch_bounds__(kTcThreads, 1) gemv_tc_kernel(const __grid_constant__ TcParams p) {
    extern __shared__ __align__(1024) unsigned char smem_raw[];
    // the swizzled activation tiles need 1024-byte aligned stages (1 KB slack is allocated)
    const uint32_t sraw = smem_u32(smem_raw);
    const uint32_t sbase = (sraw + 1023u) & ~1023u;
    unsigned char* smem = smem_raw + (sbase - sraw);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int C = p.C;
    const int u = int(blockIdx.x) / C, rank = int(blockIdx.x) - u * C;  // cluster dims (C, 1, 1)
    const int kb0 = rank * p.KB / C, nb = (rank + 1) * p.KB / C - kb0;

    // barriers: full[4] (A stage dequantized), empty[4] (stage consumed by the MMAs),
    // xfull[4] (X stage landed), acc (accumulator complete), done (every MMA finished)
    // wfull[8] / wempty[8] (weight stage landed / read by its dequantizer group)
    const uint32_t bars = sbase + p.sm_bar;
    const uint32_t bar_full = bars, bar_empty = bars + 32, bar_xfull = bars + 64, bar_acc = bars + 96,
                   bar_done = bars + 104, bar_wfull = bars + 128, bar_wempty = bars + 192;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(smem + p.sm_bar + 112);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + p.sm_bar + 116);
    const long long lim = p.wait_cycles;

    if (threadIdx.x == 0) {
        for (int a = 0; a < kTcStages; ++a) {
            mbar_init(bar_full + 8 * a, 128);
            mbar_init(bar_empty + 8 * a, 1);
            mbar_init(bar_xfull + 8 * a, 1);
        }
        mbar_init(bar_acc, 1);
        mbar_init(bar_done, 1);
        for (int w = 0; w < p.wst; ++w) {
            mbar_init(bar_wfull + 8 * w, 1);
            mbar_init(bar_wempty + 8 * w, 4);  // one arrival per warp of the consuming group
        }
        *abort = 0;
        fence_barrier_init();
    }
    const int grp = warp >> 2, r = ((warp & 3) << 5) | lane;
    const int WS = p.wst;
    const uint32_t wst0 = sbase + p.sm_w;
    // activation rows M .. n_mma are outside the tensor map: the TMA fills them with zeros
    if (warp == kTcMmaWarp) tmem_alloc(smem_u32(tmem_slot), kTcTmemCols);
    pdl_launch_dependents();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp < 8) {
        // ---------------------------------------------------------- dequantizers
        const uint32_t lane_base = tmem + (uint32_t((warp & 3) * 32) << 16);
        for (int b = grp; b < nb; b += 2) {
            const int a = b & 3, ws = b % WS;
            // the weights of block b have landed (TMA), and TMEM stage a is free again
            bool ok = tc_wait(bar_wfull + 8 * ws, (b / WS) & 1, abort, lim);
            if (ok && b >= kTcStages) ok = tc_wait(bar_empty + 8 * a, ((b >> 2) + 1) & 1, abort, lim);
            if (!__all_sync(0xffffffffu, ok)) break;  // warp-uniform: tcgen05.st is a warp-wide instruction
            tc_fence_after();
            tc_dequant<FMT>(p, r, wst0 + uint32_t(ws) * p.w_stage, lane_base + kTcACol0 + kTcACols * a);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(bar_full + 8 * a);
            __syncwarp();
            if (lane == 0) mbar_arrive(bar_wempty + 8 * ws);  // this warp has read its rows of the stage
        }
    } else if (warp == kTcXWarp) {
        // ---------------------------------------------------------- activation loader (TMA)
        pdl_wait();  // x is written by the previous kernel
        if (lane == 0) {
            const uint32_t half = uint32_t(p.n_mma) * 128u;  // one box: 64 k of every row
            int issued = 0;
            for (int b = 0; b < nb; ++b, ++issued) {
                const int a = b & 3;
                if (b >= kTcStages && !tc_wait(bar_empty + 8 * a, ((b >> 2) + 1) & 1, abort, lim)) break;
                const uint32_t xs = sbase + p.sm_x + a * (p.n_mma * 256), bar = bar_xfull + 8 * a;
                mbar_arrive_expect_tx(bar, 2u * half);
                tma_load_2d(xs, &p.xmap, (kb0 + b) * 128, 0, bar);
                tma_load_2d(xs + half, &p.xmap, (kb0 + b) * 128 + 64, 0, bar);
            }
            // no tile may still be landing when the CTA leaves (an abort skips the MMAs)
            for (int b = issued > kTcStages ? issued - kTcStages : 0; b < issued; ++b)
                tc_wait(bar_xfull + 8 * (b & 3), (b >> 2) & 1, nullptr, lim);
        }
        __syncwarp();
    } else if (warp == kTcMmaWarp) {
        // ---------------------------------------------------------- MMA issuer
        if (lane == 0) {
            bool ok = true;
            for (int b = 0; ok && b < nb; ++b) {
                const int a = b & 3;
                ok = tc_wait(bar_full + 8 * a, (b >> 2) & 1, abort, lim) &&
                     tc_wait(bar_xfull + 8 * a, (b >> 2) & 1, abort, lim);
                if (!ok) break;
                tc_fence_after();
                const uint32_t xs = sbase + p.sm_x + a * (p.n_mma * 256);
#pragma unroll
                for (int k = 0; k < 8; ++k)  // k16 step k: box k / 4, 32 B per step inside the swizzle atom
                    tc_mma(tmem, tmem + kTcACol0 + kTcACols * a + 8 * k,
                           tc_bdesc(xs + uint32_t(k >> 2) * uint32_t(p.n_mma) * 128u + 32u * uint32_t(k & 3)), p.idesc,
                           (b > 0 || k > 0) ? 1u : 0u);
                tc_commit(bar_empty + 8 * a);
            }
            if (ok) tc_commit(bar_acc);
            tc_commit(bar_done);  // every MMA issued above has finished once this completes
            tc_wait(bar_done, 0, nullptr, lim);  // also after an abort: TMEM is freed only when they are done
        }
        __syncwarp();
    } else if (warp == kTcProdWarp) {
        // ---------------------------------------------------------- weight producer (TMA)
        if (lane == 0) {
            int issued = 0;
            for (int b = 0; b < nb; ++b, ++issued) {
                const int ws = b % WS;
                if (b >= WS && !tc_wait(bar_wempty + 8 * ws, ((b / WS) + 1) & 1, abort, lim)) break;
                const uint32_t bar = bar_wfull + 8 * ws;
                mbar_arrive_expect_tx(bar, p.tx_bytes);
                tc_produce<FMT>(p, u, kb0 + b, wst0 + uint32_t(ws) * p.w_stage, bar);
            }
            // no copy may still be landing when the CTA leaves (an abort skips consumers)
            for (int b = issued > WS ? issued - WS : 0; b < issued; ++b)
                tc_wait(bar_wfull + 8 * (b % WS), (b / WS) & 1, nullptr, lim);
        }
        __syncwarp();
    } else {
        // ---------------------------------------------------------- accumulator -> shared memory
        // The X stages are free once the last MMA is done: the partial sums go there.
        const int q = warp & 3;
        const int re = (q << 5) | lane;  // TMEM lane = weight row within the unit
        const uint32_t lane_base = tmem + (uint32_t(q * 32) << 16);
        if (!epi_any(!tc_wait(bar_acc, 0, abort, lim))) {
            tc_fence_after();
            float* red = reinterpret_cast<float*>(smem + p.sm_x) + re * p.red_pitch;
            for (int mc = 0; mc < (p.n_mma >> 4); ++mc) {
                float v[16];
                tmem_ld16(lane_base + 16 * mc, v);
#pragma unroll
                for (int i = 0; i < 16; i += 4) *reinterpret_cast<float4*>(red + 16 * mc + i) = make_float4(v[i], v[i + 1], v[i + 2], v[i + 3]);
            }
        }
    }

    // ---------------------------------------------------------- cluster reduction
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    pdl_wait();  // the residual and the output are shared with the previous kernel
    cluster_sync_all();  // every CTA of the unit has its partial rows in shared memory
    int bad = 0;
    for (int c = 0; c < C; ++c) bad |= dsmem_ld_s32(dsmem_addr(smem_u32(const_cast<int*>(abort)), uint32_t(c)));
    if (!bad) {
        const bool is_silu = p.epi == BQ_EPI_SILU_MUL;
        const int half = is_silu ? 64 : 128;               // rows summed per output row: one, or the gate/up pair
        const int r0 = rank * half / C, nr = (rank + 1) * half / C - r0;
        const int mq_n = (p.M + 3) >> 2;                // groups of four activation rows
        const uint32_t red0 = sbase + p.sm_x;
        for (int t = threadIdx.x; t < nr * mq_n; t += kTcThreads) {
            const int rl = r0 + t % nr, mq = t / nr;
            const uint32_t ag = red0 + uint32_t(rl * p.red_pitch + 4 * mq) * 4u;
            const uint32_t av = red0 + uint32_t((rl + (is_silu ? 64 : 0)) * p.red_pitch + 4 * mq) * 4u;
            // every slice's partial in flight at once, then summed in rank order (deterministic)
            float4 pg[8], pu[8];
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c < C) {
                    pg[c] = c == rank ? *reinterpret_cast<const float4*>(smem + (ag - sbase)) : dsmem_ld4(dsmem_addr(ag, uint32_t(c)));
                    if (is_silu)
                        pu[c] = c == rank ? *reinterpret_cast<const float4*>(smem + (av - sbase))
                                          : dsmem_ld4(dsmem_addr(av, uint32_t(c)));
                }
            }
            float4 g = make_float4(0.f, 0.f, 0.f, 0.f), v = g;
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                if (c < C) {
                    g.x += pg[c].x; g.y += pg[c].y; g.z += pg[c].z; g.w += pg[c].w;
                    if (is_silu) {
                        v.x += pu[c].x; v.y += pu[c].y; v.z += pu[c].z; v.w += pu[c].w;
                    }
                }
            }
            const int n = tc_row(p, u, rl);
            float rs = 1.f, rsu = 1.f;
            if (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                rs = static_cast<const float*>(p.scale)[n];
                if (p.flags & BQ_FLAG_SCALE_ROUND_BF16) rs = __bfloat162float(__float2bfloat16_rn(rs));
                if (is_silu) {
                    rsu = static_cast<const float*>(p.scale)[n + (p.N >> 1)];
                    if (p.flags & BQ_FLAG_SCALE_ROUND_BF16) rsu = __bfloat162float(__float2bfloat16_rn(rsu));
                }
            }
            const float bi = p.bias ? load_act(p.bias, n, p.out_dtype) : 0.f;
            const float biu = (p.bias && is_silu) ? load_act(p.bias, n + (p.N >> 1), p.out_dtype) : 0.f;
            const float gs[4] = {g.x, g.y, g.z, g.w}, us[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int m = 4 * mq + i;
                if (m >= p.M) break;
                const float a = fmaf(gs[i], rs, bi);
                if (is_silu)
                    store_act(p.out, m * p.ldo + n, p.out_dtype, silu(a) * fmaf(us[i], rsu, biu));
                else
                    tc_store(p, m, n, a);
            }
        }
    }
    // no CTA leaves while another may still read its shared memory (every read above
    // was consumed by a store or by `bad`, so this barrier orders no memory)
    cluster_sync_relaxed();
    if (warp == kTcMmaWarp) tmem_dealloc(tmem, kTcTmemCols);
}

// RMSNorm of the activation rows into the workspace: one block per row,
// out = bf16(x * rsqrt(mean(x^2) + eps) * gamma) with fp32 math (the
// reference's rmsnorm_kernel, models/fused/kernels.py:541-557). Launched as a
// programmatic dependent: the GEMV after it starts its weight stream early.
__global__ void __launch_bounds__(256) tc_rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long long ldx,
                                                         const __nv_bfloat16* __restrict__ g,
                                                         __nv_bfloat16* __restrict__ out, int K, float eps) {
    __shared__ float red[8];
    pdl_launch_dependents();
    pdl_wait();
    const __nv_bfloat16* xr = x + blockIdx.x * ldx;
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += 256) {
        const float v = __bfloat162float(xr[k]);
        ss = fmaf(v, v, ss);
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = 1.0f / sqrtf(tot / float(K) + eps);
    __nv_bfloat16* orow = out + size_t(blockIdx.x) * K;
    for (int k = threadIdx.x; k < K; k += 256)
        orow[k] = __float2bfloat16_rn(__bfloat162float(xr[k]) * inv * __bfloat162float(g[k]));
}

const void* tc_kernel_for(int fmt) {
    switch (fmt) {
        case BQ_W_INT4_TINYGEMM: return reinterpret_cast<const void*>(gemv_tc_kernel<BQ_W_INT4_TINYGEMM>);
        case BQ_W_INT4_PLAIN: return reinterpret_cast<const void*>(gemv_tc_kernel<BQ_W_INT4_PLAIN>);
        case BQ_W_FP8_E4M3: return reinterpret_cast<const void*>(gemv_tc_kernel<BQ_W_FP8_E4M3>);
        case BQ_W_INT8: return reinterpret_cast<const void*>(gemv_tc_kernel<BQ_W_INT8>);
        case BQ_W_BF16: return reinterpret_cast<const void*>(gemv_tc_kernel<BQ_W_BF16>);
        default: return nullptr;
    }
}

}  // namespace

namespace {
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(f);
    });
    return fn;
}

// Tensor map of the activation rows: [M][K] bf16 with row stride ldx, boxes of
// 64 k x n_mma rows (rows past M read as zeros), 128-byte swizzle -- the K-major
// layout the MMA's B descriptor (tc_bdesc) describes.
int tc_encode_x(const void* x, int64_t ldx, int M, int K, int n_mma, CUtensorMap* map) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(BQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const cuuint64_t dims[2] = {cuuint64_t(K), cuuint64_t(M)};
    const cuuint64_t strides[1] = {cuuint64_t(ldx) * 2};
    const cuuint32_t box[2] = {64, cuuint32_t(n_mma)};
    const cuuint32_t es[2] = {1, 1};
    const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(x), dims, strides, box, es,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return set_error(BQ_ERR_CUDA, "cuTensorMapEncodeTiled (activations) failed (%d)", int(r));
    return BQ_OK;
}

// Tensor map of the weights, boxes of one k-block of a unit's rows (two 64-row
// boxes per k-block with SiLU*up): int4 plain rows of K/2 bytes and tinygemm's
// [N/8][K/128][8 rows][64 B] (64-byte swizzle), fp8 / int8 rows of K bytes and
// bf16 rows of K elements in 64-element halves (128-byte swizzle).
int tc_encode_weights(const bq_gemv_desc* d, CUtensorMap* map) {
    EncodeTiledFn enc = encode_fn();
    if (!enc) return set_error(BQ_ERR_CUDA, "cuTensorMapEncodeTiled is not available");
    const cuuint32_t brows = d->epilogue == BQ_EPI_SILU_MUL ? 64u : 128u;
    const cuuint32_t es[4] = {1, 1, 1, 1};
    CUresult r;
    void* w = const_cast<void*>(d->w);
    if (d->wfmt == BQ_W_INT4_TINYGEMM) {
        // [N/8][K/128][512 B]: a box is the unit's 8-row tiles of one k-block, 512 contiguous bytes each
        const cuuint64_t dims[3] = {64, cuuint64_t(d->K / 128), cuuint64_t(d->N / 8)};
        const cuuint64_t strides[2] = {512, cuuint64_t(d->K / 128) * 512};
        const cuuint32_t box[3] = {64, 1, brows / 8};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT64, 3, w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (d->wfmt == BQ_W_INT4_PLAIN) {
        const cuuint64_t dims[2] = {cuuint64_t(d->K / 2), cuuint64_t(d->N)};
        const cuuint64_t strides[1] = {cuuint64_t(d->K / 2)};
        const cuuint32_t box[2] = {64, brows};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_64B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else if (d->wfmt == BQ_W_BF16) {
        const cuuint64_t dims[2] = {cuuint64_t(d->K), cuuint64_t(d->N)};
        const cuuint64_t strides[1] = {cuuint64_t(d->K) * 2};
        const cuuint32_t box[2] = {64, brows};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    } else {
        const cuuint64_t dims[2] = {cuuint64_t(d->K), cuuint64_t(d->N)};
        const cuuint64_t strides[1] = {cuuint64_t(d->K)};
        const cuuint32_t box[2] = {128, brows};
        r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, w, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE,
                CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    }
    if (r != CUDA_SUCCESS) return set_error(BQ_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", int(r));
    return BQ_OK;
}

// Plans depend on the shape, format, group, epilogue, norm and device only.
std::mutex g_tc_mu;
std::map<std::array<int, 9>, std::pair<bool, TcPlan>> g_tc_plans;

bool plan_tc_uncached(const bq_gemv_desc* d, TcPlan* pl) {
    if (d->M < kTcMinRows || d->M > kTcMaxRows || d->x_dtype != BQ_DT_BF16 || d->N % 128 != 0) return false;
    if (d->wfmt == BQ_W_INT4_PLAIN && d->group != 128) return false;
    if (d->wfmt == BQ_W_INT4_TINYGEMM && d->group != 32 && d->group != 64 && d->group != 128 && d->group != 256)
        return false;
    const void* fn = tc_kernel_for(d->wfmt);
    if (!fn) return false;
    const DeviceInfo* di = device_info();
    if (!di) return false;
    TcPlan p{};
    p.n_mma = (d->M + 15) & ~15;
    p.KB = d->K / 128;
    p.units = d->N / 128;
    const bool int4 = d->wfmt == BQ_W_INT4_TINYGEMM || d->wfmt == BQ_W_INT4_PLAIN;
    const int ngr = int4 && d->group < 128 ? 128 / d->group : 1;
    p.w_bytes = 128u * uint32_t(tc_row_bytes(d->wfmt));
    p.tx_bytes = p.w_bytes + (int4 ? uint32_t(ngr * 512) : 0u);
    p.w_stage = (p.tx_bytes + 1023u) & ~1023u;  // swizzled boxes start on 1024-byte boundaries
    p.sm_x = 0;
    const uint32_t x_bytes = uint32_t(kTcStages) * uint32_t(p.n_mma) * 256u;
    p.sm_w = (x_bytes + 1023u) & ~1023u;
    int ws = 0;
    for (int c = std::min(kTcMaxWStages, p.KB); c >= 2; --c)
        if (p.sm_w + uint32_t(c) * p.w_stage + 256u + 1024u <= uint32_t(di->smem_optin)) {
            ws = c;
            break;
        }
    if (!ws) return false;
    p.wst = ws;
    p.sm_bar = p.sm_w + uint32_t(ws) * p.w_stage;
    p.sm_total = p.sm_bar + 256u + 1024u;  // + slack to align the layout to 1024 bytes
    p.red_pitch = uint32_t(p.n_mma) + 4u;
    if (ensure_smem_attr(fn, p.sm_total)) return false;
    // K slices per unit: fill the SMs in one wave with clusters of at most 8
    // CTAs (the portable cluster size) that can all be resident at once
    int C = std::max(1, std::min({8, p.KB, di->sm_count / std::max(1, p.units)}));
    for (; C > 1; --C) {
        cudaLaunchConfig_t cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(p.units * C);
        cfg.blockDim = dim3(kTcThreads);
        cfg.dynamicSmemBytes = p.sm_total;
        cudaLaunchAttribute at[1];
        at[0].id = cudaLaunchAttributeClusterDimension;
        at[0].val.clusterDim.x = C;
        at[0].val.clusterDim.y = 1;
        at[0].val.clusterDim.z = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, fn, &cfg) == cudaSuccess && clusters >= p.units) break;
        cudaGetLastError();  // clear a refused query
    }
    p.C = C;
    p.grid = p.units * C;
    // the normalized rows go after the arrival-counter region that every
    // workspace starts with: the row-block kernel's counters must stay zero
    p.xn_off = kCounterBytes;
    p.ws_bytes = d->gamma ? kCounterBytes + ((int64_t(d->M) * d->K * 2 + 255) & ~int64_t(255)) : 0;
    *pl = p;
    return true;
}
}  // namespace

// Plans the tensor-core path for `d`; returns false when it does not apply
// (row count, activation dtype, N, group or shared memory).
bool plan_tc(const bq_gemv_desc* d, TcPlan* pl) {
    if (d->flags & BQ_FLAG_NO_TC) return false;
    if (d->M < kTcMinRows || d->M > kTcMaxRows) return false;
    const DeviceInfo* di = device_info();
    if (!di) return false;
    const std::array<int, 9> key{di->device, d->M, d->N, d->K, d->wfmt, d->group, d->epilogue, d->x_dtype,
                                 d->gamma != nullptr ? 1 : 0};
    {
        std::lock_guard<std::mutex> lk(g_tc_mu);
        auto it = g_tc_plans.find(key);
        if (it != g_tc_plans.end()) {
            if (it->second.first) *pl = it->second.second;
            return it->second.first;
        }
    }
    TcPlan p{};
    const bool ok = plan_tc_uncached(d, &p);
    std::lock_guard<std::mutex> lk(g_tc_mu);
    if (g_tc_plans.size() > 4096) g_tc_plans.clear();
    g_tc_plans.emplace(key, std::make_pair(ok, p));
    if (ok) *pl = p;
    return ok;
}

int launch_tc(const bq_gemv_desc* d, const TcPlan& pl, void* workspace, cudaStream_t stream) {
    const void* fn = tc_kernel_for(d->wfmt);
    if (!fn) return set_error(BQ_ERR_FORMAT, "no tensor-core GEMV for format %d", d->wfmt);
    if (pl.ws_bytes > 0 && !workspace) return set_error(BQ_ERR_WORKSPACE, "the tensor-core GEMV needs a workspace");
    char* ws = static_cast<char*>(workspace);
    const __nv_bfloat16* x = static_cast<const __nv_bfloat16*>(d->x);
    long long ldx = d->ldx;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const bool pdl = (d->flags & BQ_FLAG_PDL) != 0;
    if (d->gamma) {
        __nv_bfloat16* xn = reinterpret_cast<__nv_bfloat16*>(ws + pl.xn_off);
        cudaLaunchConfig_t cfg;
        std::memset(&cfg, 0, sizeof(cfg));
        cfg.gridDim = dim3(d->M);
        cfg.blockDim = dim3(256);
        cfg.stream = stream;
        if (pdl) {
            cfg.attrs = attr;
            cfg.numAttrs = 1;
        }
        const __nv_bfloat16* g = static_cast<const __nv_bfloat16*>(d->gamma);
        const int K = d->K;
        const float eps = d->eps;
        void* args[] = {&x, &ldx, &g, &xn, const_cast<int*>(&K), const_cast<float*>(&eps)};
        cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(tc_rmsnorm_kernel), args);
        if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "RMSNorm launch failed: %s", cudaGetErrorString(e));
        x = xn;
        ldx = d->K;
    } else if ((reinterpret_cast<uintptr_t>(x) & 15) || (ldx * 2) % 16) {
        return set_error(BQ_ERR_ALIGN, "the tensor-core GEMV needs 16-byte aligned activation rows");
    }
    TcParams p;
    std::memset(&p, 0, sizeof(p));
    {
        const int rc = tc_encode_x(x, ldx, d->M, d->K, pl.n_mma, &p.xmap);
        if (rc) return rc;
    }
    p.w = d->w;
    p.scale = d->scale;
    p.bias = d->bias;
    p.residual = d->residual;
    p.out = d->out;
    p.x = x;
    p.ldx = ldx;
    p.ldr = d->ldr;
    p.ldo = d->ldo;
    p.M = d->M;
    p.N = d->N;
    p.K = d->K;
    p.KB = pl.KB;
    p.group = d->group;
    p.epi = d->epilogue;
    p.out_dtype = d->out_dtype;
    p.res_dtype = d->res_dtype;
    p.flags = d->flags;
    p.C = pl.C;
    p.n_mma = pl.n_mma;
    p.wst = pl.wst;
    // kind::f16, fp32 accumulate, bf16 A and B, both K-major, N = n_mma, M = 128
    p.idesc = (1u << 4) | (1u << 7) | (1u << 10) | (uint32_t(pl.n_mma >> 3) << 17) | (uint32_t(128 >> 4) << 24);
    p.wait_cycles = kWaitCycles;
    p.sm_x = pl.sm_x;
    p.sm_w = pl.sm_w;
    p.sm_bar = pl.sm_bar;
    p.sm_total = pl.sm_total;
    p.red_pitch = pl.red_pitch;
    p.w_stage = pl.w_stage;
    p.w_bytes = pl.w_bytes;
    p.tx_bytes = pl.tx_bytes;
    {
        const int rc = tc_encode_weights(d, &p.wmap);
        if (rc) return rc;
    }
    int rc = ensure_smem_attr(fn, pl.sm_total);
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kTcThreads);
    cfg.dynamicSmemBytes = pl.sm_total;
    cfg.stream = stream;
    int na = 0;
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = pl.C;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    if (pdl || d->gamma) ++na;  // after the norm kernel always: its rows are waited for in the kernel
    cfg.attrs = (pdl || d->gamma) ? attr : attr + 1;
    cfg.numAttrs = na + 1;
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "tensor-core GEMV launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // namespace bq
