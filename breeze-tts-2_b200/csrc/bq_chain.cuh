// Decode chain: a list of GEMVs (one decode step's projections) in ONE
// persistent cooperative launch, one CTA per SM.
//
//  * Warp 8 of every CTA is a producer: it walks the op list and streams the
//    weights of every tile this CTA owns, chunk by chunk, into a ring of
//    shared-memory slots with 1-D bulk copies that complete on mbarriers
//    (full[s] / empty[s]). It runs ahead of the compute across op
//    boundaries, limited only by the ring, so the weight stream does not
//    stop at the end of an op; the next ops' weights are already on chip
//    when their inputs become ready.
//  * Warps 0-7 consume. For op j they wait until op j-1 is complete -- a
//    per-op counter in global memory that every CTA increments once per op
//    (epoch-based targets, so counters never need resetting between
//    launches) -- then load x (L2 only: other CTAs wrote it during this
//    launch), stage it per warp (RMSNorm's gamma arrives through the ring),
//    run the same in-register dequantization and m16n8k16 tensor-core dot
//    products as bq_gemv on each chunk, reduce the eight warps' partial sums
//    in shared memory, apply the epilogue and store. No grid barrier: a CTA
//    waits only for the op whose output it reads.
//  * Tiles are 16 output rows (SiLU*up: 16 gate + 16 up rows); op j's tile t
//    belongs to CTA (base_j + t) % grid, base_j rotating so every CTA gets an
//    even share of the step's weight bytes. A chunk is a tile x a K range.
//  * Every wait is bounded; on a timeout the kernel sets the device error
//    bit, every CTA stops at its next wait, the producer waits (bounded) for
//    its copies in flight, and the kernel returns. The counters are then
//    inconsistent: bq_gemv_chain_prepare must run again before a new launch.
#pragma once

#include <cuda_runtime.h>

#include "bq_device.cuh"
#include "bq_gemv3.cuh"
#include "bq_host.h"

namespace bq {

constexpr int kChainWarps = 8;                      // consumer warps
constexpr int kChainThreads = (kChainWarps + 1) * 32;  // + the producer warp
constexpr int kChainMaxTiles = 4;                   // tiles one CTA may own in one op
constexpr int kCounterStride = 32;                  // 128 bytes between per-op counters

// One GEMV of the chain (device copy written by bq_gemv_chain_prepare).
struct ChainOp {
    int32_t fmt, M, N, K, KB, group, gpk, epi, norm;
    int32_t x_dtype, out_dtype, res_dtype;
    uint32_t flags;
    float eps;
    int32_t n_half;       // SiLU: N / 2
    int32_t tiles;        // tiles of 16 rows (SiLU: gate/up pairs)
    int32_t pieces;       // 16-row pieces per tile: 1, or 2 (SiLU)
    int32_t nchunk;       // K chunks per tile
    int32_t kbc;          // k-blocks (128 k) per chunk
    int32_t base;         // tile t -> CTA (base + t) % grid
    uint32_t piece_bytes; // ring bytes of one piece of a chunk: weights, then scales (16-aligned)
    uint32_t wpiece;      // weight bytes of one piece of a chunk
    uint32_t chunk_bytes; // pieces * piece_bytes
    int32_t row_copies;   // bulk copies per piece for the weights (1, 2 or 16)
    const void* x;
    int64_t ldx;
    const void* w;
    const void* scale;    // int4: tile-major copy [N/16][K/g][16][2] bf16; fp8/int8: [N] fp32
    const void* gamma;
    const void* bias;
    const void* residual;
    int64_t ldr;
    void* out;
    int64_t ldo;
};

// Workspace header (written by bq_gemv_chain_prepare, kept up to date by the kernel).
struct ChainHeader {
    unsigned int epoch;  // launches completed
    unsigned int pad0[7];
    long long wait_cycles;
    const unsigned int* start_flag;
    unsigned int start_target;
    unsigned int pad1[19];
    unsigned int finish;  // CTAs finished in the current launch (offset 128)
};

struct ChainArgs {
    const ChainOp* ops;
    int32_t n_ops;
    int32_t ring_slots;
    uint32_t slot_bytes;
    uint32_t smem_x, smem_xsum, smem_part, smem_misc, smem_bar;
    uint32_t xw_bytes;     // staged activations per warp (M rows + a zero block)
    uint32_t xw_pitch;     // bytes per staged row
    uint32_t xsum_w_bytes; // int4 group sums per warp: [block][sub-group][16 rows] fp32
    uint32_t part_bytes;   // partial sums of one tile (the area holds kChainMaxTiles of them)
    unsigned int* counters;  // [n_ops][kCounterStride]
    ChainHeader* hdr;
};

// ---------------------------------------------------------------- sync helpers
__device__ __forceinline__ unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void consumer_sync() { asm volatile("bar.sync 1, 256;" ::: "memory"); }
// Barrier of the consumer warps that also ORs a flag over them: every
// consumer thread gets the same answer, so a decision taken on it (stop
// after an abort) is uniform and no warp is left waiting at a later barrier.
__device__ __forceinline__ bool consumer_sync_or(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred p, q;\n\t"
        "setp.ne.u32 q, %1, 0;\n\t"
        "bar.red.or.pred p, 1, 256, q;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(r)
        : "r"(uint32_t(v))
        : "memory");
    return r != 0;
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// 1-D bulk copy global -> shared, completion counted in bytes on an mbarrier
// (16-byte aligned addresses, size a multiple of 16; no multicast).
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
                 ::"r"(dst), "l"(src), "r"(bytes), "r"(bar)
                 : "memory");
}

// Shared abort state of one CTA: once any wait of the CTA gives up, or the
// device error word is set by another CTA, every later wait returns at once.
struct ChainCtl {
    volatile int abort;
    long long limit;  // bound of every wait, SM cycles
};

__device__ __forceinline__ bool chain_aborted(ChainCtl* ctl) {
    if (ctl->abort) return true;
    if (*reinterpret_cast<volatile unsigned int*>(&g_device_error) != 0u) {
        ctl->abort = 1;
        return true;
    }
    return false;
}

// Bounded mbarrier wait; false (and the CTA aborts) on timeout or abort.
// backoff_ns > 0: sleep between polls (the producer's waits for a free slot,
// so its spinning does not take issue slots from the consumer warps).
__device__ __forceinline__ bool chain_mbar_wait(uint32_t bar, uint32_t parity, ChainCtl* ctl, int backoff_ns) {
    const long long limit = ctl->limit;
    if (mbar_try_wait(bar, parity)) return true;
    const long long t0 = clock64();
    int spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if (backoff_ns > 0) __nanosleep(backoff_ns);
        if ((++spins & 255) == 0) {
            if (chain_aborted(ctl)) return false;
            if (clock64() - t0 > limit) {
                atomicOr(&g_device_error, BQ_DEVERR_WAIT_TIMEOUT_BIT);
                ctl->abort = 1;
                return false;
            }
        }
    }
    return true;
}

// Bounded wait for a global counter to reach `target` (wrap-safe); one
// thread. SYS: the word may be written by the host (system-scope acquire).
template <bool SYS = false>
__device__ __forceinline__ bool chain_counter_wait(const unsigned int* c, unsigned int target, ChainCtl* ctl) {
    const long long limit = ctl->limit;
    auto load = [&]() { return SYS ? ld_acquire_sys(c) : ld_acquire_gpu(c); };
    if (int(load() - target) >= 0) return true;
    const long long t0 = clock64();
    int spins = 0;
    while (int(load() - target) < 0) {
        if ((++spins & 63) == 0) {
            if (chain_aborted(ctl)) return false;
            if (clock64() - t0 > limit) {
                atomicOr(&g_device_error, BQ_DEVERR_WAIT_TIMEOUT_BIT);
                ctl->abort = 1;
                return false;
            }
        }
    }
    return true;
}

// Tiles of op `op` owned by CTA `cta`: t = first + i * grid.
__device__ __forceinline__ int chain_first_tile(const ChainOp& op, int cta, int grid) {
    const int r = (cta - op.base) % grid;
    return r < 0 ? r + grid : r;
}

// Global row of piece p of tile t.
__device__ __forceinline__ int chain_piece_row(const ChainOp& op, int t, int p) {
    return op.epi == BQ_EPI_SILU_MUL ? (p == 0 ? 16 * t : op.n_half + 16 * t) : 16 * t;
}

// Weight bytes per row per k-block.
__device__ __forceinline__ int chain_row_kb_bytes(int fmt) {
    return fmt == BQ_W_BF16 ? 256 : (fmt == BQ_W_FP8_E4M3 || fmt == BQ_W_INT8) ? 128 : 64;
}

// ---------------------------------------------------------------- producer
// Streams, for every op in order, the gamma of a normed op and then every
// chunk of every tile this CTA owns into the ring. `q` counts ring uses;
// the consumers walk the same sequence.
__device__ __forceinline__ void chain_producer(const ChainArgs& a, uint8_t* smem, ChainCtl* ctl) {
    const int lane = threadIdx.x & 31;
    const int cta = blockIdx.x, grid = gridDim.x;
    const uint32_t ring = smem_u32(smem);
    const uint32_t bars = smem_u32(smem + a.smem_bar);  // full[R] then empty[R], 8 bytes each
    const int R = a.ring_slots;
    uint32_t q = 0, s = 0, phase = 0;  // fills issued; next slot and the parity of its current fill
    bool ok = true;
    auto acquire_slot = [&](uint32_t bytes, uint32_t& dst, uint32_t& full) -> bool {
        // lane 0 decides for the warp, so every lane takes the same path
        int free_slot = 0;
        if (lane == 0) free_slot = chain_mbar_wait(bars + 8u * (R + s), phase ^ 1u, ctl, 128) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, free_slot, 0)) return false;
        dst = ring + s * a.slot_bytes;
        full = bars + 8u * s;
        if (lane == 0) mbar_arrive_expect_tx(full, bytes);
        __syncwarp();
        ++q;
        if (++s == uint32_t(R)) {
            s = 0;
            phase ^= 1u;
        }
        return true;
    };
    for (int j = 0; j < a.n_ops && ok; ++j) {
        const ChainOp op = a.ops[j];  // private copy, as in the consumers
        const int t0 = chain_first_tile(op, cta, grid);
        if (t0 >= op.tiles) continue;
        uint32_t dst, full;
        if (op.norm) {
            if (!(ok = acquire_slot(uint32_t(op.K) * 2u, dst, full))) break;
            if (lane == 0) bulk_g2s(dst, op.gamma, uint32_t(op.K) * 2u, full);
        }
        const int rkb = chain_row_kb_bytes(op.fmt);
        const bool int4 = op.fmt == BQ_W_INT4_TINYGEMM || op.fmt == BQ_W_INT4_PLAIN;
        const bool rowscale = op.fmt == BQ_W_FP8_E4M3 || op.fmt == BQ_W_INT8;
        const int groups_per_chunk = (op.kbc * kKB) / op.group;  // int4 group rows per chunk (group <= kbc*128)
        for (int t = t0; t < op.tiles && ok; t += grid) {
            for (int c = 0; c < op.nchunk; ++c) {
                const uint32_t wbytes = op.wpiece, sbytes = int4 ? uint32_t(groups_per_chunk) * 64u : (rowscale ? 64u : 0u);
                if (!(ok = acquire_slot(uint32_t(op.pieces) * (wbytes + sbytes), dst, full))) break;
                for (int p = 0; p < op.pieces; ++p) {
                    const int row0 = chain_piece_row(op, t, p);
                    const uint32_t pb = dst + uint32_t(p) * op.piece_bytes;
                    const uint8_t* w = static_cast<const uint8_t*>(op.w);
                    // weights: copy i of this piece is issued by lane i
                    if (op.fmt == BQ_W_INT4_TINYGEMM) {
                        if (lane < 2) {
                            const uint32_t nb = uint32_t(op.kbc) * 512u;
                            bulk_g2s(pb + uint32_t(lane) * nb,
                                     w + ((int64_t(row0 / 8 + lane) * op.KB + int64_t(c) * op.kbc) * 512), nb, full);
                        }
                    } else {
                        const int64_t row_bytes = int64_t(op.KB) * rkb;
                        if (op.nchunk == 1) {
                            if (lane == 0) bulk_g2s(pb, w + int64_t(row0) * row_bytes, wbytes, full);
                        } else if (lane < 16) {
                            const uint32_t nb = uint32_t(op.kbc) * uint32_t(rkb);
                            bulk_g2s(pb + uint32_t(lane) * nb,
                                     w + int64_t(row0 + lane) * row_bytes + int64_t(c) * op.kbc * rkb, nb, full);
                        }
                    }
                    if (lane == 31 && sbytes) {
                        const uint8_t* sc = static_cast<const uint8_t*>(op.scale);
                        const uint8_t* src = int4 ? sc + (int64_t(row0 / 16) * (op.K / op.group) +
                                                          int64_t(c) * groups_per_chunk) * 64
                                                  : sc + int64_t(row0) * 4;
                        bulk_g2s(pb + wbytes, src, sbytes, full);
                    }
                }
            }
        }
    }
    // Wait (bounded) for the copies in flight in every slot before leaving:
    // the last use of each slot is its only pending fill.
    const uint32_t first = q > uint32_t(R) ? q - uint32_t(R) : 0u;
    for (uint32_t u = first; u < q && lane == 0; ++u) {
        const uint32_t s = u % uint32_t(R);
        const long long t0 = clock64();
        while (!mbar_try_wait(bars + 8u * s, (u / uint32_t(R)) & 1u)) {
            if (clock64() - t0 > ctl->limit) {
                atomicOr(&g_device_error, BQ_DEVERR_WAIT_TIMEOUT_BIT);
                break;
            }
        }
    }
}

// ---------------------------------------------------------------- consumers
// Per-warp view of one op: warp w takes k-blocks [lo, lo + cnt) of every
// chunk; over the op's chunks that is nkw = nchunk * cnt blocks, staged as
// local blocks j = c * cnt + i (global k-block c * kbc + lo + i).
struct ChainWarpK {
    int lo, cnt, nkw;
    __device__ __forceinline__ int global_kb(const ChainOp& op, int j) const {
        const int c = cnt ? j / cnt : 0;
        return c * op.kbc + lo + (j - c * cnt);
    }
};

__device__ __forceinline__ ChainWarpK chain_warp_k(const ChainOp& op, int warp) {
    ChainWarpK k;
    k.lo = (warp * op.kbc) >> 3;
    k.cnt = (((warp + 1) * op.kbc) >> 3) - k.lo;
    k.nkw = op.nchunk * k.cnt;
    return k;
}

// Misc area (floats): ss[8 warps][16 rows], up[8][16], rscale[kChainMaxTiles][2
// pieces][16], then the residual rows of the CTA's tiles (bf16
// [kChainMaxTiles][16 rows of M][16 columns]).
struct ChainMisc {
    float* ss;
    float* up;
    float* rscale;
    __nv_bfloat16* res;
};
__device__ __forceinline__ ChainMisc chain_misc(const ChainArgs& a, uint8_t* smem) {
    float* f = reinterpret_cast<float*>(smem + a.smem_misc);
    return ChainMisc{f, f + 128, f + 256, reinterpret_cast<__nv_bfloat16*>(f + 256 + kChainMaxTiles * 32)};
}
constexpr uint32_t chain_misc_bytes() { return (256 + kChainMaxTiles * 32) * 4 + kChainMaxTiles * 16 * 16 * 2; }

// Staging of this warp's activations after its x copies landed: bf16 x*gamma
// in place for int4 / bf16 weights (sum of x^2 per row kept per lane, reduced
// across the row's lanes), f16 scaled by a per-(warp, row) power of two for
// fp8 / int8 (exact conversions of the weights), as bq_gemv stages them. For
// int4 weights the same pass sums the staged (bf16-rounded) activations of
// every group: xs[(j * GPK + sg) * 16 + m], the X of the group term
// s * (C - (128 + offset) X) + z * X. Local block j = c * cnt + i holds global
// k-block c * kbc + lo + i; the loops walk chunks and blocks without divisions.
template <int FMT, int GPK>
__device__ __forceinline__ void chain_stage(const ChainOp& op, const ChainWarpK& wk, uint8_t* xw, uint32_t pitch,
                                            const uint8_t* gam, ChainMisc& mc, float* xs, int warp, int lane) {
    using F = Fmt3<FMT>;
    const int M = op.M;
    const bool norm = op.norm != 0;
    int lg = 0;
    while ((1 << lg) < M) ++lg;
    const int kp_log = 5 - lg, kp = 1 << kp_log;  // lanes per row
    const int lm = lane >> kp_log, lk = lane & (kp - 1);
    const bool rowok = lm < M;
    uint8_t* xrow = xw + lm * pitch;
    // unit u (8 values) of the warp's blocks: local block u >> 4, 8 values at (u & 15) * 8.
    // Lane lk of a row takes units lk, lk + kp, ...: with kp >= 16 one pass covers
    // kp / 16 blocks, else 16 / kp passes cover one block.
    const int units = 16 * wk.nkw;
    const int upb = kp >= 16 ? 16 : kp;  // lanes of one block within a row group
    auto gkb = [&](int j) { return (j / (wk.cnt > 0 ? wk.cnt : 1)) * op.kbc + wk.lo + j % (wk.cnt > 0 ? wk.cnt : 1); };
    float ss_lane = 0.f;
    if constexpr (!F::kF16) {
        const bool identity = FMT != BQ_W_INT4_PLAIN && !norm && !F::kInt4;
        float xg[GPK];
#pragma unroll
        for (int g = 0; g < GPK; ++g) xg[g] = 0.f;
        if (!identity) {
            // warp-uniform trip count (the group-sum shuffles need every lane)
#pragma unroll 1
            for (int base = 0; base < units; base += kp) {
                const int u = base + lk;
                const bool ok = rowok && u < units;
                const int j = u >> 4, off = j * 256 + (u & 15) * 16;
                float v[8];
                if (ok) {
                    const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                    v[0] = bf16lo(r.x); v[1] = bf16hi(r.x); v[2] = bf16lo(r.y); v[3] = bf16hi(r.y);
                    v[4] = bf16lo(r.z); v[5] = bf16hi(r.z); v[6] = bf16lo(r.w); v[7] = bf16hi(r.w);
                } else {
#pragma unroll
                    for (int e = 0; e < 8; ++e) v[e] = 0.f;
                }
                if (norm && ok) {
                    const uint4 gv = *reinterpret_cast<const uint4*>(gam + (gkb(j) * 128 + (u & 15) * 8) * 2);
                    const float g8[8] = {bf16lo(gv.x), bf16hi(gv.x), bf16lo(gv.y), bf16hi(gv.y),
                                         bf16lo(gv.z), bf16hi(gv.z), bf16lo(gv.w), bf16hi(gv.w)};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        ss_lane = fmaf(v[e], v[e], ss_lane);
                        v[e] *= g8[e];
                    }
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
                if (ok && (norm || FMT == BQ_W_INT4_PLAIN)) *reinterpret_cast<uint4*>(xrow + off) = o;
                if constexpr (F::kInt4) {
                    // this unit's share of its group: the rounded values the MMAs read
                    const float part = ((bf16lo(o.x) + bf16hi(o.x)) + (bf16lo(o.y) + bf16hi(o.y))) +
                                       ((bf16lo(o.z) + bf16hi(o.z)) + (bf16lo(o.w) + bf16hi(o.w)));
                    xg[GPK == 1 ? 0 : ((u & 15) * GPK) >> 4] += part;
                    // a block is complete for this row group after its last unit: reduce
                    // over the lanes that share it and store the row's X
                    const bool last = kp >= 16 ? true : ((u & 15) + kp >= 16);
                    if (last) {
#pragma unroll
                        for (int g = 0; g < GPK; ++g) {
                            float t = xg[g];
                            for (int o2 = 1; o2 < upb; o2 <<= 1) t += __shfl_xor_sync(0xffffffffu, t, o2);
                            xg[g] = 0.f;
                            if (ok && (lk & (upb - 1)) == 0) xs[(j * GPK + g) * 16 + lm] = t;
                        }
                    }
                }
            }
        }
        if (norm) {
            for (int o2 = kp >> 1; o2; o2 >>= 1) ss_lane += __shfl_xor_sync(0xffffffffu, ss_lane, o2);
            if (lk == 0 && rowok) mc.ss[warp * 16 + lm] = ss_lane;
        }
    } else {
        float ss = 0.f, amax = 0.f;
        if (rowok) {
#pragma unroll 2
            for (int u = lk; u < units; u += kp) {
                const int j = u >> 4, off = j * 256 + (u & 15) * 16;
                const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                const float v[8] = {bf16lo(r.x), bf16hi(r.x), bf16lo(r.y), bf16hi(r.y),
                                    bf16lo(r.z), bf16hi(r.z), bf16lo(r.w), bf16hi(r.w)};
                float g8[8] = {1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f, 1.f};
                if (norm) {
                    const uint4 gv = *reinterpret_cast<const uint4*>(gam + (gkb(j) * 128 + (u & 15) * 8) * 2);
                    g8[0] = bf16lo(gv.x); g8[1] = bf16hi(gv.x); g8[2] = bf16lo(gv.y); g8[3] = bf16hi(gv.y);
                    g8[4] = bf16lo(gv.z); g8[5] = bf16hi(gv.z); g8[6] = bf16lo(gv.w); g8[7] = bf16hi(gv.w);
                }
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    ss = fmaf(v[e], v[e], ss);
                    amax = fmaxf(amax, fabsf(v[e] * g8[e]));
                }
            }
        }
        for (int o2 = kp >> 1; o2; o2 >>= 1) {
            ss += __shfl_xor_sync(0xffffffffu, ss, o2);
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o2));
        }
        int e = 0;
        if (amax > 0.f && amax < INFINITY) {
            int ex;
            frexpf(amax, &ex);
            e = min(max(ex - 15, -100), 100);
        }
        const float down = __int_as_float((127 - e) << 23);
        if (lk == 0 && rowok) {
            mc.ss[warp * 16 + lm] = ss;
            mc.up[warp * 16 + lm] = __int_as_float((127 + e) << 23);
        }
        if (rowok) {
#pragma unroll 2
            for (int u = lk; u < units; u += kp) {
                const int j = u >> 4, off = j * 256 + (u & 15) * 16;
                const uint4 r = *reinterpret_cast<const uint4*>(xrow + off);
                float v[8] = {bf16lo(r.x), bf16hi(r.x), bf16lo(r.y), bf16hi(r.y),
                              bf16lo(r.z), bf16hi(r.z), bf16lo(r.w), bf16hi(r.w)};
                if (norm) {
                    const uint4 gv = *reinterpret_cast<const uint4*>(gam + (gkb(j) * 128 + (u & 15) * 8) * 2);
                    v[0] *= bf16lo(gv.x); v[1] *= bf16hi(gv.x); v[2] *= bf16lo(gv.y); v[3] *= bf16hi(gv.y);
                    v[4] *= bf16lo(gv.z); v[5] *= bf16hi(gv.z); v[6] *= bf16lo(gv.w); v[7] *= bf16hi(gv.w);
                }
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
}

// Activation fragments (B operand) of staged local block j, per M tile.
template <int FMT, int MT>
__device__ __forceinline__ void chain_bfrag(const uint8_t* xw, uint32_t xw_s, uint32_t pitch, int M, int j, int lane,
                                            const uint8_t* xzero, uint32_t xzero_s, uint32_t (&bfr)[MT][16]) {
    const int tq = lane & 3, tg = lane >> 2;
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
            const int m = 8 * mt + (lane & 7);
            const int koff = ((lane >> 4) * 16) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t a = m < M ? xw_s + m * pitch + (j * 128 + q * 32 + koff) * 2 : xzero_s;
                asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                             : "=r"(bfr[mt][4 * q]), "=r"(bfr[mt][4 * q + 1]), "=r"(bfr[mt][4 * q + 2]),
                               "=r"(bfr[mt][4 * q + 3])
                             : "r"(a)
                             : "memory");
            }
        } else {
            const int m = 8 * mt + tg;
            const uint8_t* row = m < M ? xw + m * pitch + j * 256 : xzero;
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
}

// One chunk of one tile: this warp's k-blocks [wk.lo, wk.lo + wk.cnt) of the
// chunk in ring slot `slot`, accumulated into acc[piece][mt]. Local staged
// block index of the first one: j0.
template <int FMT, int MT, int GPK>
__device__ __forceinline__ void chain_chunk(const ChainOp& op, const uint8_t* slot, const ChainWarpK& wk, int j0,
                                            const uint8_t* xw, uint32_t xw_s, uint32_t pitch, const uint8_t* xzero,
                                            uint32_t xzero_s, const float* xs, int lane, float (&acc)[2][MT][4]) {
    using F = Fmt3<FMT>;
    constexpr int NCH = MT == 1 ? 4 : 2;  // independent MMA chains
    const int tq = lane & 3, tg = lane >> 2;
    const int rkb = chain_row_kb_bytes(FMT);
    const uint32_t rs = uint32_t(op.kbc) * uint32_t(rkb);  // row stride of a row-major piece
#pragma unroll 2
    for (int i = 0; i < wk.cnt; ++i) {
        const int ic = wk.lo + i;  // block within the chunk
        uint32_t bfr[MT][16];
        chain_bfrag<FMT, MT>(xw, xw_s, pitch, op.M, j0 + i, lane, xzero, xzero_s, bfr);
        float sA[GPK][MT][2], sX[GPK][MT][2];
        if constexpr (F::kInt4) {
            constexpr float kMagic = 128.f + float(F::kOfs);  // dequantized code = 128 + q
#pragma unroll
            for (int sg = 0; sg < GPK; ++sg)
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const int m0 = 8 * mt + 2 * tq;
                    const float2 xx = *reinterpret_cast<const float2*>(xs + ((j0 + i) * GPK + sg) * 16 + m0);
                    sX[sg][mt][0] = m0 < op.M ? xx.x : 0.f;
                    sX[sg][mt][1] = m0 + 1 < op.M ? xx.y : 0.f;
                    sA[sg][mt][0] = kMagic * sX[sg][mt][0];
                    sA[sg][mt][1] = kMagic * sX[sg][mt][1];
                }
        }
#pragma unroll
        for (int p = 0; p < 2; ++p) {
            if (p >= op.pieces) continue;
            const uint8_t* pb = slot + p * op.piece_bytes;
            if constexpr (F::kInt4) {
                uint4 r0, r1;
                if constexpr (FMT == BQ_W_INT4_TINYGEMM) {
                    r0 = *reinterpret_cast<const uint4*>(pb + ic * 512 + lane * 16);
                    r1 = *reinterpret_cast<const uint4*>(pb + op.kbc * 512 + ic * 512 + lane * 16);
                } else {
                    r0 = *reinterpret_cast<const uint4*>(pb + tg * rs + ic * 64 + tq * 16);
                    r1 = *reinterpret_cast<const uint4*>(pb + (tg + 8) * rs + ic * 64 + tq * 16);
                }
                const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                const uint8_t* szs = pb + op.wpiece;
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
                            mma_bf16(c2[ii % NCH][mt], a0, a1, a2, a3, bfr[mt][2 * ki], bfr[mt][2 * ki + 1]);
                    }
#pragma unroll
                    for (int h = 1; h < NCH; ++h)
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                            for (int d = 0; d < 4; ++d) c2[0][mt][d] += c2[h][mt][d];
                    // scale/zero rows of this group: 64 bytes (16 rows x {s, z}) each
                    const int gr = op.group >= 128 ? (ic * kKB) / op.group : ic * GPK + sg;
                    const uint32_t sz0 = *reinterpret_cast<const uint32_t*>(szs + gr * 64 + tg * 4);
                    const uint32_t sz1 = *reinterpret_cast<const uint32_t*>(szs + gr * 64 + (tg + 8) * 4);
                    const float s0 = bf16lo(sz0), z0 = bf16hi(sz0), s1 = bf16lo(sz1), z1 = bf16hi(sz1);
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt) {
                        float* a = acc[p][mt];
                        a[0] += s0 * (c2[0][mt][0] - sA[sg][mt][0]) + z0 * sX[sg][mt][0];
                        a[1] += s0 * (c2[0][mt][1] - sA[sg][mt][1]) + z0 * sX[sg][mt][1];
                        a[2] += s1 * (c2[0][mt][2] - sA[sg][mt][0]) + z1 * sX[sg][mt][0];
                        a[3] += s1 * (c2[0][mt][3] - sA[sg][mt][1]) + z1 * sX[sg][mt][1];
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
                    const uint4 r0 = *reinterpret_cast<const uint4*>(pb + tg * rs + ic * rkb + b * 64 + tq * 16);
                    const uint4 r1 = *reinterpret_cast<const uint4*>(pb + (tg + 8) * rs + ic * rkb + b * 64 + tq * 16);
                    const uint32_t w0[4] = {r0.x, r0.y, r0.z, r0.w};
                    const uint32_t w1[4] = {r1.x, r1.y, r1.z, r1.w};
                    if constexpr (FMT == BQ_W_BF16) {
#pragma unroll
                        for (int e2 = 0; e2 < 2; ++e2) {
                            const int ki = 2 * b + e2;
#pragma unroll
                            for (int mt = 0; mt < MT; ++mt)
                                mma_bf16(c2[ki % NCH][mt], w0[2 * e2], w1[2 * e2], w0[2 * e2 + 1], w1[2 * e2 + 1],
                                         bfr[mt][2 * ki], bfr[mt][2 * ki + 1]);
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
                                mma_f16(c2[ki % NCH][mt], a0, a1, a2, a3, bfr[mt][2 * ki], bfr[mt][2 * ki + 1]);
                        }
                    }
                }
#pragma unroll
                for (int h = 0; h < NCH; ++h)
#pragma unroll
                    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                        for (int d = 0; d < 4; ++d) acc[p][mt][d] += c2[h][mt][d];
            }
        }
    }
}

// Reduction over the eight warps, norm factor, row scale, bias and the
// epilogue of one tile, for the M tile `mt` (one warp per M tile).
template <int FMT, int MT>
__device__ __forceinline__ void chain_epilogue(const ChainOp& op, const float4* part, const ChainMisc& mc, int t,
                                               int ti, int mt, int lane) {
    using F = Fmt3<FMT>;
    const int tq = lane & 3, tg = lane >> 2;
    const int M = op.M;
    const int nq = M >= 7 ? 4 : (M + 1) >> 1;
    float v[2][4];
#pragma unroll
    for (int p = 0; p < 2; ++p) {
        float4 qv[8];
#pragma unroll
        for (int w = 0; w < 8; ++w)
            qv[w] = (p < op.pieces && tq < nq) ? part[((((w * 2 + p) * MT + mt) * 8 + tg) * nq + tq)]
                                               : make_float4(0.f, 0.f, 0.f, 0.f);
        v[p][0] = ((qv[0].x + qv[1].x) + (qv[2].x + qv[3].x)) + ((qv[4].x + qv[5].x) + (qv[6].x + qv[7].x));
        v[p][1] = ((qv[0].y + qv[1].y) + (qv[2].y + qv[3].y)) + ((qv[4].y + qv[5].y) + (qv[6].y + qv[7].y));
        v[p][2] = ((qv[0].z + qv[1].z) + (qv[2].z + qv[3].z)) + ((qv[4].z + qv[5].z) + (qv[6].z + qv[7].z));
        v[p][3] = ((qv[0].w + qv[1].w) + (qv[2].w + qv[3].w)) + ((qv[4].w + qv[5].w) + (qv[6].w + qv[7].w));
    }
    const int m0 = 8 * mt + 2 * tq;
    float inv0 = 1.f, inv1 = 1.f;
    if (op.norm) {
        float s2 = 0.f;
        if (lane < M) {
#pragma unroll
            for (int w = 0; w < 8; ++w) s2 += mc.ss[w * 16 + lane];
        }
        const float invl = rsqrtf(s2 / float(op.K) + op.eps);
        inv0 = __shfl_sync(0xffffffffu, invl, m0 & 31);
        inv1 = __shfl_sync(0xffffffffu, invl, (m0 + 1) & 31);
    }
#pragma unroll
    for (int p = 0; p < 2; ++p)
#pragma unroll
        for (int d = 0; d < 4; ++d) {
            const int r = tg + (d >> 1) * 8;
            float sc = 1.f;
            if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) sc = mc.rscale[(ti * 2 + p) * 16 + r];
            float o = v[p][d] * ((d & 1) ? inv1 : inv0) * sc;
            if (op.bias && p < op.pieces) o += load_act(op.bias, chain_piece_row(op, t, p) + r, op.out_dtype);
            v[p][d] = o;
        }
#pragma unroll
    for (int d = 0; d < 4; ++d) {
        const int r = tg + (d >> 1) * 8, m = m0 + (d & 1);
        if (m >= M) continue;
        const int n = 16 * t + r;
        if (op.epi == BQ_EPI_SILU_MUL) {
            store_act(op.out, int64_t(m) * op.ldo + n, op.out_dtype, silu(v[0][d]) * v[1][d]);
        } else {
            float o = v[0][d];
            if (op.epi == BQ_EPI_ADD_RESIDUAL) o += __bfloat162float(mc.res[(ti * 16 + m) * 16 + r]);
            store_act(op.out, int64_t(m) * op.ldo + n, op.out_dtype, o);
        }
    }
}

// Ring position of the consumers: slot index and the parity of its current fill.
struct ChainRing {
    uint32_t slot, phase;
    __device__ __forceinline__ void advance(int R) {
        if (++slot == uint32_t(R)) {
            slot = 0;
            phase ^= 1u;
        }
    }
};

// One op's work on this CTA's tiles (consumer warps; the op's inputs are ready).
// Every warp computes its k-blocks of every tile, chunk by chunk as they land,
// and leaves each tile's partial sums in shared memory; after one barrier the
// warps reduce and store the tiles in parallel, one (tile, M tile) each.
template <int FMT, int MT, int GPK>
__device__ __forceinline__ void chain_op_body(const ChainArgs& a, const ChainOp& op, uint8_t* smem, ChainCtl* ctl,
                                              ChainRing& ring) {
    using F = Fmt3<FMT>;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int tq = lane & 3, tg = lane >> 2;
    const int grid = gridDim.x, M = op.M, R = a.ring_slots;
    const uint32_t bars = smem_u32(smem + a.smem_bar);
    ChainMisc mc = chain_misc(a, smem);
    const ChainWarpK wk = chain_warp_k(op, warp);
    uint8_t* xw = smem + a.smem_x + warp * a.xw_bytes;
    const uint32_t xw_s = smem_u32(xw);
    const uint8_t* xzero = xw + M * a.xw_pitch;
    const uint32_t xzero_s = smem_u32(xzero);
    float* xs = reinterpret_cast<float*>(smem + a.smem_xsum + warp * a.xsum_w_bytes);
    const int t0 = chain_first_tile(op, blockIdx.x, grid);
    const int ntile = (op.tiles - t0 + grid - 1) / grid;

    // x (this warp's blocks) and the residual rows of the CTA's tiles: L2 only
    if (wk.cnt > 0) {
        const char* xb = static_cast<const char*>(op.x);
        const int per_row = wk.nkw * 16;
        for (int sidx = lane; sidx < M * per_row; sidx += 32) {
            const int m = sidx / per_row, r = sidx - m * per_row;
            const int jl = r >> 4, c = jl / wk.cnt, kb = c * op.kbc + wk.lo + (jl - c * wk.cnt);
            cp_async16(xw_s + m * a.xw_pitch + jl * 256 + (r & 15) * 16,
                       xb + (int64_t(m) * op.ldx + kb * 128 + (r & 15) * 8) * 2);
        }
    }
    if (op.epi == BQ_EPI_ADD_RESIDUAL) {
        const char* rb = static_cast<const char*>(op.residual);
        for (int c = threadIdx.x; c < ntile * M * 2; c += kChainWarps * 32) {
            const int ti = c / (M * 2), r = c - ti * M * 2, m = r >> 1, h = r & 1;
            const int n = 16 * (t0 + ti * grid) + 8 * h;
            cp_async16(smem_u32(mc.res + (ti * 16 + m) * 16 + 8 * h), rb + (int64_t(m) * op.ldr + n) * 2);
        }
    }
    cp_async_commit();
    // gamma arrives through the ring ahead of the weights
    uint32_t gslot = 0;
    const uint8_t* gam = nullptr;
    if (op.norm) {
        gslot = ring.slot;
        chain_mbar_wait(bars + 8u * gslot, ring.phase, ctl, 0);
        ring.advance(R);
        gam = smem + gslot * a.slot_bytes;
    }
    asm volatile("cp.async.wait_group 0;" ::: "memory");
    __syncwarp();
    chain_stage<FMT, GPK>(op, wk, xw, a.xw_pitch, gam, mc, xs, warp, lane);
    if (op.norm && lane == 0) mbar_arrive(bars + 8u * (R + gslot));

    const int nq = M >= 7 ? 4 : (M + 1) >> 1;
#pragma unroll 1
    for (int ti = 0; ti < ntile; ++ti) {
        float acc[2][MT][4];
#pragma unroll
        for (int p = 0; p < 2; ++p)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int d = 0; d < 4; ++d) acc[p][mt][d] = 0.f;
#pragma unroll 1
        for (int c = 0; c < op.nchunk; ++c) {
            const uint32_t sl = ring.slot;
            chain_mbar_wait(bars + 8u * sl, ring.phase, ctl, 0);
            ring.advance(R);
            const uint8_t* slot = smem + sl * a.slot_bytes;
            chain_chunk<FMT, MT, GPK>(op, slot, wk, c * wk.cnt, xw, xw_s, a.xw_pitch, xzero, xzero_s, xs, lane, acc);
            if constexpr (FMT == BQ_W_FP8_E4M3 || FMT == BQ_W_INT8) {
                if (c == op.nchunk - 1 && warp == 0 && lane < 16 * op.pieces) {
                    const int p = lane >> 4;
                    float sc = *reinterpret_cast<const float*>(slot + p * op.piece_bytes + op.wpiece + (lane & 15) * 4);
                    if (FMT == BQ_W_INT8 && (op.flags & BQ_FLAG_SCALE_ROUND_BF16)) sc = __bfloat162float(__float2bfloat16_rn(sc));
                    mc.rscale[(ti * 2 + p) * 16 + (lane & 15)] = sc;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(bars + 8u * (R + sl));
        }
        float4* part = reinterpret_cast<float4*>(smem + a.smem_part + ti * a.part_bytes);
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            const int m0 = 8 * mt + 2 * tq;
            const float u0 = m0 < M ? (F::kF16 ? mc.up[warp * 16 + m0] : 1.f) : 0.f;
            const float u1 = m0 + 1 < M ? (F::kF16 ? mc.up[warp * 16 + m0 + 1] : 1.f) : 0.f;
#pragma unroll
            for (int p = 0; p < 2; ++p)
                if (p < op.pieces && tq < nq)
                    part[(((warp * 2 + p) * MT + mt) * 8 + tg) * nq + tq] =
                        make_float4(acc[p][mt][0] * u0, acc[p][mt][1] * u1, acc[p][mt][2] * u0, acc[p][mt][3] * u1);
        }
    }
    consumer_sync();
    for (int task = warp; task < ntile * MT; task += kChainWarps) {
        const int ti = task / MT, mt = task - ti * MT;
        chain_epilogue<FMT, MT>(op, reinterpret_cast<const float4*>(smem + a.smem_part + ti * a.part_bytes), mc,
                                t0 + ti * grid, ti, mt, lane);
    }
}

// FMT >= 0: every op of the chain has this format (and GPK): one body, a
// small kernel whose code stays in the instruction caches from op to op (the
// all-format kernel spent ~1 us per op refetching its code). FMT < 0: any
// mix of formats, dispatched per op.
template <int MT, int FMT, int GPK>
__device__ __forceinline__ void chain_dispatch(const ChainArgs& a, const ChainOp& op, uint8_t* smem, ChainCtl* ctl,
                                               ChainRing& ring) {
    if constexpr (FMT >= 0) {
        chain_op_body<FMT, MT, GPK>(a, op, smem, ctl, ring);
        return;
    }
    switch (op.fmt) {
        case BQ_W_INT4_TINYGEMM:
            if (op.gpk == 4)
                chain_op_body<BQ_W_INT4_TINYGEMM, MT, 4>(a, op, smem, ctl, ring);
            else if (op.gpk == 2)
                chain_op_body<BQ_W_INT4_TINYGEMM, MT, 2>(a, op, smem, ctl, ring);
            else
                chain_op_body<BQ_W_INT4_TINYGEMM, MT, 1>(a, op, smem, ctl, ring);
            break;
        case BQ_W_INT4_PLAIN: chain_op_body<BQ_W_INT4_PLAIN, MT, 1>(a, op, smem, ctl, ring); break;
        case BQ_W_FP8_E4M3: chain_op_body<BQ_W_FP8_E4M3, MT, 1>(a, op, smem, ctl, ring); break;
        case BQ_W_INT8: chain_op_body<BQ_W_INT8, MT, 1>(a, op, smem, ctl, ring); break;
        default: chain_op_body<BQ_W_BF16, MT, 1>(a, op, smem, ctl, ring); break;
    }
}

// Consumer warps: every op in order. A CTA that owns tiles of op j waits for
// op j - 1 (or the start flag), works, and signals op j once all its stores
// are issued and fenced; a CTA with no tiles in op j signals at once (it
// reads and writes nothing for it).
template <int MT, int FMT, int GPK>
__device__ __forceinline__ void chain_consumer(const ChainArgs& a, const ChainHeader* hdr, uint8_t* smem,
                                               ChainCtl* ctl, unsigned int target) {
    ChainRing ring{0u, 0u};
    // the waiting and signalling thread sits in warp 1: warp 0 shares its
    // scheduler with the producer warp
    constexpr int kLead = 32;
    for (int j = 0; j < a.n_ops; ++j) {
        // a private copy: the inline-PTX memory clobbers of the hot loops would
        // otherwise make every field a fresh global load
        const ChainOp op = a.ops[j];
        if (chain_first_tile(op, blockIdx.x, gridDim.x) < op.tiles) {
            if (threadIdx.x == kLead) {
                if (j > 0)
                    chain_counter_wait(a.counters + (j - 1) * kCounterStride, target, ctl);
                else if (hdr->start_flag)
                    chain_counter_wait<true>(hdr->start_flag, hdr->start_target, ctl);
                __threadfence();
            }
            if (consumer_sync_or(ctl->abort != 0)) return;
            chain_dispatch<MT, FMT, GPK>(a, op, smem, ctl, ring);
            if (consumer_sync_or(ctl->abort != 0)) return;
        }
        if (threadIdx.x == kLead) {
            __threadfence();
            atomicAdd(a.counters + j * kCounterStride, 1u);
        }
    }
}

template <int MT, int FMT, int GPK>
__global__ void __launch_bounds__(kChainThreads, 1) gemv_chain_kernel(const ChainArgs a) {
    extern __shared__ __align__(1024) uint8_t smem[];
    __shared__ ChainCtl ctl;
    __shared__ unsigned int s_epoch;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    ChainHeader* hdr = a.hdr;
    if (threadIdx.x == 0) {
        ctl.abort = 0;
        ctl.limit = hdr->wait_cycles > 0 ? hdr->wait_cycles : kWaitCycles;
        const uint32_t bars = smem_u32(smem + a.smem_bar);
        for (int s = 0; s < a.ring_slots; ++s) {
            mbar_init(bars + 8u * s, 1u);
            mbar_init(bars + 8u * (a.ring_slots + s), uint32_t(kChainWarps));
        }
        fence_barrier_init();
    }
    if (warp < kChainWarps && lane < 16)  // the zero block after each warp's staged rows
        reinterpret_cast<uint4*>(smem + a.smem_x + warp * a.xw_bytes + a.ops[0].M * a.xw_pitch)[lane] =
            make_uint4(0u, 0u, 0u, 0u);
    pdl_launch_dependents();
    pdl_wait();  // the first op's inputs may come from the preceding kernel
    if (threadIdx.x == 0) s_epoch = *reinterpret_cast<volatile unsigned int*>(&hdr->epoch);
    __syncthreads();
    if (warp == kChainWarps)
        chain_producer(a, smem, &ctl);
    else
        chain_consumer<MT, FMT, GPK>(a, hdr, smem, &ctl, (s_epoch + 1u) * gridDim.x);
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(&hdr->finish, 1u) == gridDim.x - 1) {
            hdr->finish = 0u;
            __threadfence();
            atomicExch(&hdr->epoch, s_epoch + 1u);
        }
    }
}

}  // namespace bq
