// Decode attention step for sm_100a (bq_attention_step): per-head q/k RMSNorm,
// RoPE, KV-cache write and split-sequence flash-decode with the combine
// fused into the same launch (the last CTA of a (row, kv head) to finish
// merges the splits, fixed order). Replaces qkv_rope_cache_kernel,
// attn_decode_kernel and attn_combine_kernel (models/fused/kernels.py:376-536).
//
// Grid (splits, HKV, B), 128 threads. A CTA owns one kv head of one batch
// row and a contiguous slice of the cache positions [0, pos]; it computes its
// G = HQ / HKV query heads and the new k / v itself, so no CTA reads the
// cache at `pos` before it is written (the split holding `pos` uses the new
// values from registers and is the one that writes them back).
#include <cooperative_groups.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

namespace {

constexpr int kAttnThreads = 128;
constexpr int kMaxG = 8;  // query heads per kv head
// Fixed counter region at the start of the workspace (one counter per (row,
// kv head)): a shape-dependent size would let one call's partials land where
// a later call with more (row, kv head) pairs keeps its counters.
constexpr int kAttnMaxPairs = 4096;
constexpr size_t kAttnCounterBytes = size_t(kAttnMaxPairs) * 4;
constexpr int kAttnOMaxB = 4;    // batch rows of the fused attention + O step
constexpr int kAttnOMaxS = 256;  // its cache length (every chunk recomputes the attention)
constexpr int kAttnOMaxR = 64;   // its output rows per CTA

struct AttnParams {
    int32_t B, HQ, HKV, S, G, splits, mask_dtype, has_norm;
    float eps, scale;
    const __nv_bfloat16* qkv;
    int64_t ldqkv;
    const __nv_bfloat16* cos;
    const __nv_bfloat16* sin;
    int64_t ldcs;
    const int64_t* pos;
    __nv_bfloat16* kc;
    __nv_bfloat16* vc;
    const void* mask;
    int64_t ldm;
    const __nv_bfloat16* qn;
    const __nv_bfloat16* kn;
    __nv_bfloat16* out;
    int64_t ldo;
    unsigned int* counters;  // [B][HKV]
    float* partials;         // [B][HKV][splits][G][D + 2]
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Lane holds dims [lane * DPL, lane * DPL + DPL). Per-head RMSNorm (optional)
// and RoPE with rotate_half: the partner of dim i is i +- D/2, held by
// lane ^ 16.
template <int DPL>
__device__ __forceinline__ void norm_rope(float (&v)[DPL], const __nv_bfloat16* w, float eps, bool norm,
                                          const float (&c)[DPL], const float (&s)[DPL], int lane) {
    constexpr int D = 32 * DPL;
    if (norm) {
        float ss = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) ss += v[e] * v[e];
        ss = warp_sum(ss);
        const float inv = 1.0f / sqrtf(ss / float(D) + eps);
#pragma unroll
        for (int e = 0; e < DPL; ++e) v[e] = v[e] * inv * __bfloat162float(w[lane * DPL + e]);
    }
    float rot[DPL];
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
        const float partner = __shfl_xor_sync(0xffffffffu, v[e], 16);
        rot[e] = lane < 16 ? -partner : partner;
    }
#pragma unroll
    for (int e = 0; e < DPL; ++e) v[e] = v[e] * c[e] + rot[e] * s[e];
}

template <int DPL>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[DPL]) {
    if constexpr (DPL == 4) {
        const uint2 r = *reinterpret_cast<const uint2*>(p);
        v[0] = __uint_as_float(r.x << 16);
        v[1] = __uint_as_float(r.x & 0xFFFF0000u);
        v[2] = __uint_as_float(r.y << 16);
        v[3] = __uint_as_float(r.y & 0xFFFF0000u);
    } else {
        const uint32_t r = *reinterpret_cast<const uint32_t*>(p);
        v[0] = __uint_as_float(r << 16);
        v[1] = __uint_as_float(r & 0xFFFF0000u);
    }
}

// This lane's pieces of the step's inputs that do not depend on the cache
// position: cos / sin, the warp's query heads, and (on the k / v warp) the new
// k and v -- loaded right after the dependent-launch wait, together with the
// position itself, so the chain pays one round trip for all of them.
constexpr int kQPW = (kMaxG + 3) / 4;  // query heads per warp at most
template <int DPL>
struct AttnIn {
    float c[DPL], s[DPL];
    float q[kQPW][DPL];
    float k[DPL];
    __nv_bfloat16 v[DPL];
};

// The warp that owns the new k / v: one without a query head when G < 4, so
// it runs beside the q heads.
__device__ __forceinline__ int attn_kv_warp(int G) { return G < 4 ? G : 3; }

template <int DPL>
__device__ __forceinline__ void attn_load(const AttnParams& p, int j, int b, AttnIn<DPL>& in) {
    constexpr int D = 32 * DPL;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G;
    const __nv_bfloat16* cp = p.cos + int64_t(b) * p.ldcs + lane * DPL;
    const __nv_bfloat16* sn = p.sin + int64_t(b) * p.ldcs + lane * DPL;
#pragma unroll
    for (int e = 0; e < DPL; ++e) {
        in.c[e] = __bfloat162float(cp[e]);
        in.s[e] = __bfloat162float(sn[e]);
    }
    const __nv_bfloat16* row = p.qkv + int64_t(b) * p.ldqkv;
#pragma unroll
    for (int gi = 0; gi < kQPW; ++gi) {
        const int g = warp + 4 * gi;
        if (g < G) {
            const __nv_bfloat16* q = row + (j * G + g) * D + lane * DPL;
#pragma unroll
            for (int e = 0; e < DPL; ++e) in.q[gi][e] = __bfloat162float(q[e]);
        }
    }
    if (warp == attn_kv_warp(G)) {
        const __nv_bfloat16* k = row + (p.HQ + j) * D + lane * DPL;
        const __nv_bfloat16* vv = row + (p.HQ + p.HKV + j) * D + lane * DPL;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            in.k[e] = __bfloat162float(k[e]);
            in.v[e] = vv[e];
        }
    }
}

// One kv head of one batch row over the cache positions [s_lo, s_hi): the
// query heads and the new k (normed, roped, rounded to the cache dtype) and v
// (from `in`) into shared memory, the new k / v into the caches when
// `holds_pos` (register copies stand in for position pos, so nothing reads it
// before it is written), then each warp's online-softmax state over its
// positions in s_red. Ends with a block barrier. (Requesting the warp's first
// batch of cache rows before the q / k work as well measured slower on the
// depth frame: 4649 -> 5212 us.)
template <int DPL>
__device__ __forceinline__ void attn_core(const AttnParams& p, int j, int b, int64_t pos, int s_lo, int s_hi,
                                          bool holds_pos, const AttnIn<DPL>& in, float (*s_q)[32 * DPL], float* s_k,
                                          float* s_v, float (*s_red)[kMaxG][32 * DPL + 2]) {
    constexpr int D = 32 * DPL;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G;
    // query heads of this kv head, scaled by D^-0.5 (kept in fp32, as the reference's q buffer)
#pragma unroll
    for (int gi = 0; gi < kQPW; ++gi) {
        const int g = warp + 4 * gi;
        if (g < G) {
            float v[DPL];
#pragma unroll
            for (int e = 0; e < DPL; ++e) v[e] = in.q[gi][e];
            norm_rope<DPL>(v, p.qn, p.eps, p.has_norm, in.c, in.s, lane);
#pragma unroll
            for (int e = 0; e < DPL; ++e) s_q[g][lane * DPL + e] = v[e] * p.scale;
        }
    }
    // the new k (normed, roped, rounded to the cache dtype) and v
    if (warp == attn_kv_warp(G)) {
        float v[DPL];
#pragma unroll
        for (int e = 0; e < DPL; ++e) v[e] = in.k[e];
        norm_rope<DPL>(v, p.kn, p.eps, p.has_norm, in.c, in.s, lane);
        const int64_t at = ((int64_t(b) * p.HKV + j) * p.S + pos) * D + lane * DPL;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            const __nv_bfloat16 kb = __float2bfloat16_rn(v[e]);
            s_k[lane * DPL + e] = __bfloat162float(kb);
            s_v[lane * DPL + e] = __bfloat162float(in.v[e]);
            if (holds_pos) {
                p.kc[at + e] = kb;
                p.vc[at + e] = in.v[e];
            }
        }
    }
    __syncthreads();

    // ---- online softmax over this split's positions; warp w takes s = s_lo + w (mod 4)
    float qr[kMaxG][DPL], m[kMaxG], l[kMaxG], acc[kMaxG][DPL];
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        m[g] = -1e30f;
        l[g] = 0.f;
#pragma unroll
        for (int e = 0; e < DPL; ++e) {
            qr[g][e] = g < G ? s_q[g][lane * DPL + e] : 0.f;
            acc[g][e] = 0.f;
        }
    }
    const int64_t kv_base = (int64_t(b) * p.HKV + j) * p.S * D + lane * DPL;
    // Batches of PB positions per warp (warp w takes s_lo + w + 4 * (PB * it + i)):
    // all k / v rows of a batch are loaded before any is used, then one
    // online-softmax update per head covers the batch.
    constexpr int PB = 4;
    for (int t0 = s_lo + warp; t0 < s_hi; t0 += 4 * PB) {
        float kr[PB][DPL], vr[PB][DPL], mk[PB];
        bool ok[PB];
#pragma unroll
        for (int i = 0; i < PB; ++i) {
            const int t = t0 + 4 * i;
            ok[i] = t < s_hi;
            const int tt = ok[i] ? t : t0;  // a row that exists; its result is discarded
            if (tt == pos) {
#pragma unroll
                for (int e = 0; e < DPL; ++e) {
                    kr[i][e] = s_k[lane * DPL + e];
                    vr[i][e] = s_v[lane * DPL + e];
                }
            } else {
                load_row<DPL>(p.kc + kv_base + int64_t(tt) * D, kr[i]);
                load_row<DPL>(p.vc + kv_base + int64_t(tt) * D, vr[i]);
            }
            mk[i] = 0.f;
            if (p.mask) {
                mk[i] = p.mask_dtype == BQ_DT_BF16
                            ? __bfloat162float(static_cast<const __nv_bfloat16*>(p.mask)[int64_t(b) * p.ldm + tt])
                            : static_cast<const float*>(p.mask)[int64_t(b) * p.ldm + tt];
            }
        }
#pragma unroll
        for (int g = 0; g < kMaxG; ++g) {
            if (g >= G) break;
            float sc[PB];
#pragma unroll
            for (int i = 0; i < PB; ++i) {
                float d = 0.f;
#pragma unroll
                for (int e = 0; e < DPL; ++e) d = fmaf(qr[g][e], kr[i][e], d);
                sc[i] = d;
            }
#pragma unroll
            for (int o = 16; o; o >>= 1)
#pragma unroll
                for (int i = 0; i < PB; ++i) sc[i] += __shfl_xor_sync(0xffffffffu, sc[i], o);
            float bm = m[g];
#pragma unroll
            for (int i = 0; i < PB; ++i) {
                sc[i] = ok[i] ? sc[i] + mk[i] : -1e30f;
                bm = fmaxf(bm, sc[i]);
            }
            const float alpha = __expf(m[g] - bm);
            float ls = l[g] * alpha;
            float a2[DPL];
#pragma unroll
            for (int e = 0; e < DPL; ++e) a2[e] = acc[g][e] * alpha;
#pragma unroll
            for (int i = 0; i < PB; ++i) {
                const float pr = ok[i] ? __expf(sc[i] - bm) : 0.f;
                ls += pr;
#pragma unroll
                for (int e = 0; e < DPL; ++e) a2[e] = fmaf(pr, vr[i][e], a2[e]);
            }
            l[g] = ls;
#pragma unroll
            for (int e = 0; e < DPL; ++e) acc[g][e] = a2[e];
            m[g] = bm;
        }
    }
    // ---- merge the 4 warps
#pragma unroll
    for (int g = 0; g < kMaxG; ++g) {
        if (g >= G) break;
#pragma unroll
        for (int e = 0; e < DPL; ++e) s_red[warp][g][lane * DPL + e] = acc[g][e];
        if (lane == 0) {
            s_red[warp][g][D] = m[g];
            s_red[warp][g][D + 1] = l[g];
        }
    }
    __syncthreads();
}

// CLUSTER (1 < splits <= 8): the splits of one (row, kv head) form a
// thread-block cluster; each keeps its (acc, m, l) per head in shared memory and
// every CTA combines a slice of the output dimensions over all splits through
// distributed shared memory, in split order (the same arithmetic and order as
// the global combine, so the results agree bit for bit): no global partials,
// fences or arrival counters.
template <int DPL, bool CLUSTER>
__global__ void __launch_bounds__(kAttnThreads) attention_step_kernel(const AttnParams p) {
    constexpr int D = 32 * DPL;
    __shared__ float s_q[kMaxG][D];
    __shared__ float s_k[D], s_v[D];
    __shared__ float s_red[4][kMaxG][D + 2];
    __shared__ float s_split[CLUSTER ? kMaxG : 1][D + 2];  // cluster mode: this split's (acc, m, l) per head
    __shared__ unsigned int s_last;
    const int sp = blockIdx.x, j = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = p.G;

    // Before the dependent-launch wait: pull this CTA's slice of the caches into
    // L2 (positions before the current one do not depend on the preceding
    // kernel). The position read here is only a hint; it is read again below.
    if (threadIdx.x == 0) {
        const int64_t hint = *reinterpret_cast<const volatile int64_t*>(p.pos);
        if (hint >= 0 && hint < p.S) {
            const int len = int(hint) + 1, per0 = (len + p.splits - 1) / p.splits;
            const int lo = sp * per0, hi = min(lo + per0, len);
            if (hi > lo) {
                const int64_t base = ((int64_t(b) * p.HKV + j) * p.S + lo) * D;
                const uint32_t bytes = uint32_t(hi - lo) * D * 2;
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.kc + base), "r"(bytes) : "memory");
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p.vc + base), "r"(bytes) : "memory");
            }
        }
    }
    pdl_wait();  // qkv comes from the preceding projection

    AttnIn<DPL> in;
    attn_load<DPL>(p, j, b, in);  // in flight together with the position
    const int64_t pos = *p.pos;
    if (pos < 0 || pos >= p.S) {  // a position outside the cache: flag it, touch nothing
        if (threadIdx.x == 0 && sp == 0 && j == 0 && b == 0) atomicOr(&g_device_error, BQ_DEVERR_POSITION_BIT);
        return;
    }
    const int kv_len = int(pos) + 1;
    const int per = (kv_len + p.splits - 1) / p.splits;
    const int s_lo = sp * per, s_hi = min(s_lo + per, kv_len);
    const bool holds_pos = pos >= s_lo && pos < s_hi;

    attn_core<DPL>(p, j, b, pos, s_lo, s_hi, holds_pos, in, s_q, s_k, s_v, s_red);
    // the next launch starts once this step's cache reads are done (decode step with
    // attention, int4 M=1: 1017 -> 980 us; the fused attention + O kernel keeps its
    // trigger before the wait: the depth frame measured slower the other way)
    pdl_launch_dependents();
    // thread t < G * D: (head g, dim d); fixed warp order
    const float* red = &s_red[0][0][0];
    constexpr int HS = kMaxG * (D + 2);  // stride between warps
    for (int t = threadIdx.x; t < G * D; t += kAttnThreads) {
        const int g = t / D, d = t - g * D;
        float mm = -1e30f;
#pragma unroll
        for (int w = 0; w < 4; ++w) mm = fmaxf(mm, red[w * HS + g * (D + 2) + D]);
        float ll = 0.f, aa = 0.f;
#pragma unroll
        for (int w = 0; w < 4; ++w) {
            const float f = __expf(red[w * HS + g * (D + 2) + D] - mm);
            ll += red[w * HS + g * (D + 2) + D + 1] * f;
            aa += red[w * HS + g * (D + 2) + d] * f;
        }
        if (p.splits == 1) {
            p.out[int64_t(b) * p.ldo + (j * G + g) * D + d] = __float2bfloat16_rn(aa / ll);
        } else if constexpr (CLUSTER) {
            s_split[g][d] = aa;
            if (d == 0) {
                s_split[g][D] = mm;
                s_split[g][D + 1] = ll;
            }
        } else {
            float* part = p.partials + (((int64_t(b) * p.HKV + j) * p.splits + sp) * G + g) * (D + 2);
            __stcg(part + d, aa);
            if (d == 0) {
                __stcg(part + D, mm);
                __stcg(part + D + 1, ll);
            }
        }
    }
    if (p.splits == 1) return;
    if constexpr (CLUSTER) {
        cluster_sync_all();  // every split's (acc, m, l) is in its shared memory
        // split sp (= cluster rank) finishes output elements [sp GD / splits, (sp + 1) GD / splits)
        const int GD = G * D, lo = sp * GD / p.splits, hi = (sp + 1) * GD / p.splits;
        for (int t = lo + threadIdx.x; t < hi; t += kAttnThreads) {
            const int g = t / D, d = t - g * D;
            const uint32_t a0 = smem_u32(&s_split[g][0]);
            float mq[8], lq[8], aq[8];
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (q < p.splits) {
                    const uint32_t aq_ = dsmem_addr(a0, uint32_t(q));
                    mq[q] = dsmem_ld_f32(aq_ + uint32_t(D * 4));
                    lq[q] = dsmem_ld_f32(aq_ + uint32_t((D + 1) * 4));
                    aq[q] = dsmem_ld_f32(aq_ + uint32_t(d * 4));
                }
            }
            float mm = -1e30f;
#pragma unroll
            for (int q = 0; q < 8; ++q)
                if (q < p.splits) mm = fmaxf(mm, mq[q]);
            float ll = 0.f, aa = 0.f;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                if (q < p.splits) {
                    const float f = __expf(mq[q] - mm);
                    ll += lq[q] * f;
                    aa += aq[q] * f;
                }
            }
            p.out[int64_t(b) * p.ldo + (j * G + g) * D + d] = __float2bfloat16_rn(aa / ll);
        }
        // the peers' buffers stay until read (the reads were consumed by the stores above)
        cluster_sync_relaxed();
        return;
    }
    // ---- the last split to finish merges all splits (fixed order)
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned int old = atomicAdd(p.counters + b * p.HKV + j, 1u);
        s_last = old == unsigned(p.splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = p.partials + ((int64_t(b) * p.HKV + j) * p.splits) * G * (D + 2);
    for (int t = threadIdx.x; t < G * D; t += kAttnThreads) {
        const int g = t / D, d = t - g * D;
        float mm = -1e30f;
        for (int q = 0; q < p.splits; ++q) mm = fmaxf(mm, __ldcg(base + (q * G + g) * (D + 2) + D));
        float ll = 0.f, aa = 0.f;
        for (int q = 0; q < p.splits; ++q) {
            const float* pq = base + (q * G + g) * (D + 2);
            const float f = __expf(__ldcg(pq + D) - mm);
            ll += __ldcg(pq + D + 1) * f;
            aa += __ldcg(pq + d) * f;
        }
        p.out[int64_t(b) * p.ldo + (j * G + g) * D + d] = __float2bfloat16_rn(aa / ll);
    }
    if (threadIdx.x == 0) atomicExch(p.counters + b * p.HKV + j, 0u);
}

// ---------------------------------------------------------------- attention + O projection
// The attention step fused with the output projection and its residual add
// (out = residual + attn @ Wo^T), for short caches. CTA (c, j, b) owns kv head
// j of batch row b and the R output rows [c R, c R + R): before the
// dependent-launch wait it stages its slice of Wo (R rows x the G D columns of
// head j's query heads); after it, it computes head j's attention for row b
// (each chunk recomputes it, cheap at these lengths; chunk 0 writes the
// caches), rounds it to bf16 as the unfused step stores it, and writes its
// fp32 partial rows. The last of the HKV CTAs of (chunk, row) sums the heads
// in head order, adds the residual and stores bf16.
struct AttnOParams {
    AttnParams a;          // splits = 1; a.out unused
    int32_t R, pad;        // output rows per CTA
    const __nv_bfloat16* wo;
    int64_t ldw;
    const __nv_bfloat16* res;
    int64_t ldr;
    __nv_bfloat16* out;
    int64_t ldo;
    unsigned int* counters;  // [N / R][B]
    float* partials;         // [N / R][B][HKV][R]
};

// CLUSTER: the HKV CTAs of one (chunk, row) form a thread-block cluster
// (HKV <= 8); the partial rows stay in shared memory and each CTA sums its
// share of the rows over the heads through distributed shared memory, with
// no global partials, fences or arrival counters.
template <int DPL, bool CLUSTER>
__global__ void __launch_bounds__(kAttnThreads) attention_o_kernel(const AttnOParams p) {
    constexpr int D = 32 * DPL;
    __shared__ float s_part[kAttnOMaxR];  // cluster mode: this head's partial rows
    __shared__ float s_q[kMaxG][D];
    __shared__ float s_k[D], s_v[D];
    __shared__ float s_red[4][kMaxG][D + 2];
    __shared__ unsigned int s_last;
    extern __shared__ __align__(16) uint8_t attn_o_dsm[];
    const AttnParams& a = p.a;
    const int c = blockIdx.x, j = blockIdx.y, b = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int G = a.G, GD = a.G * D, R = p.R;
    const __nv_bfloat16* s_w = reinterpret_cast<const __nv_bfloat16*>(attn_o_dsm);  // [R][GD]
    float* s_o = reinterpret_cast<float*>(attn_o_dsm + size_t(R) * GD * 2);        // [GD]

    // before the wait: the static Wo slice, and an L2 hint for this head's cache rows
    {
        const int per_row = GD / 8;  // 16-byte pieces
        const uint32_t w0 = smem_u32(attn_o_dsm);
        for (int i = threadIdx.x; i < R * per_row; i += kAttnThreads) {
            const int r = i / per_row, q = i - r * per_row;
            cp_async16(w0 + uint32_t(r * GD * 2 + q * 16), p.wo + (int64_t(c) * R + r) * p.ldw + int64_t(j) * GD + q * 8);
        }
    }
    if (threadIdx.x == 0) {
        const int64_t hint = *reinterpret_cast<const volatile int64_t*>(a.pos);
        if (hint >= 0 && hint < a.S) {
            const uint32_t bytes = uint32_t(hint + 1) * D * 2;
            const int64_t base = (int64_t(b) * a.HKV + j) * a.S * D;
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.kc + base), "r"(bytes) : "memory");
            asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(a.vc + base), "r"(bytes) : "memory");
        }
    }
    pdl_launch_dependents();
    pdl_wait();  // qkv and the residual come from preceding kernels

    AttnIn<DPL> in;
    attn_load<DPL>(a, j, b, in);  // in flight together with the position
    const int64_t pos = *a.pos;
    if (pos < 0 || pos >= a.S) {  // a position outside the cache: flag it, touch nothing
        cp_async_wait_all();
        if (threadIdx.x == 0 && c == 0 && j == 0 && b == 0) atomicOr(&g_device_error, BQ_DEVERR_POSITION_BIT);
        return;
    }
    const int kv_len = int(pos) + 1;
    const float* red = &s_red[0][0][0];
    constexpr int HS = kMaxG * (D + 2);  // stride between warps
    // the residual of the first output row this thread finishes, in flight during the attention
    const int r_first = CLUSTER ? j + a.HKV * int(threadIdx.x) : int(threadIdx.x);
    const float res_first =
        r_first < R ? __bfloat162float(p.res[int64_t(b) * p.ldr + int64_t(c) * R + r_first]) : 0.f;
    {
        attn_core<DPL>(a, j, b, pos, 0, kv_len, c == 0, in, s_q, s_k, s_v, s_red);
        for (int t = threadIdx.x; t < GD; t += kAttnThreads) {
            const int g = t / D, d = t - g * D;
            float mm = -1e30f;
#pragma unroll
            for (int w = 0; w < 4; ++w) mm = fmaxf(mm, red[w * HS + g * (D + 2) + D]);
            float ll = 0.f, aa = 0.f;
#pragma unroll
            for (int w = 0; w < 4; ++w) {
                const float f = __expf(red[w * HS + g * (D + 2) + D] - mm);
                ll += red[w * HS + g * (D + 2) + D + 1] * f;
                aa += red[w * HS + g * (D + 2) + d] * f;
            }
            s_o[t] = __bfloat162float(__float2bfloat16_rn(aa / ll));
        }
    }
    cp_async_wait_all();  // this thread's pieces of the Wo slice
    __syncthreads();

    // partial rows: warp w takes rows w, w + 4, ...; lanes split the G D columns
    const int64_t cb = int64_t(c) * a.B + b;  // (chunk, row)
    float* part = CLUSTER ? s_part : p.partials + (cb * a.HKV + j) * R;
    // four rows at a time with independent accumulators and reductions (R is a multiple of 16)
    for (int r0 = warp; r0 < R; r0 += 16) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        for (int t = lane * 2; t < GD; t += 64) {
            const float o0 = s_o[t], o1 = s_o[t + 1];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                const uint32_t w2 = *reinterpret_cast<const uint32_t*>(s_w + (r0 + 4 * q) * GD + t);
                acc[q] = fmaf(__uint_as_float(w2 << 16), o0, acc[q]);
                acc[q] = fmaf(__uint_as_float(w2 & 0xFFFF0000u), o1, acc[q]);
            }
        }
#pragma unroll
        for (int q = 0; q < 4; ++q) acc[q] = warp_sum(acc[q]);
        if (lane == 0) {
#pragma unroll
            for (int q = 0; q < 4; ++q) {
                if constexpr (CLUSTER)
                    part[r0 + 4 * q] = acc[q];
                else
                    __stcg(part + r0 + 4 * q, acc[q]);
            }
        }
    }
    if constexpr (CLUSTER) {
        namespace cg = cooperative_groups;
        cg::cluster_group cluster = cg::this_cluster();
        cluster.sync();  // every head's partial rows are in its shared memory
        // cluster rank = kv head j; this CTA finishes rows j, j + HKV, ...
        for (int r = j + a.HKV * int(threadIdx.x); r < R; r += a.HKV * kAttnThreads) {
            float v = 0.f;
            for (int h = 0; h < a.HKV; ++h) v += cluster.map_shared_rank(s_part, h)[r];
            const int64_t n = int64_t(c) * R + r;
            v += r == r_first ? res_first : __bfloat162float(p.res[int64_t(b) * p.ldr + n]);
            p.out[int64_t(b) * p.ldo + n] = __float2bfloat16_rn(v);
        }
        // no CTA leaves while another may still read its partials (every read above
        // was consumed by its store, so the barrier needs no memory ordering)
        cluster_sync_relaxed();
        return;
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(p.counters + cb, 1u) == unsigned(a.HKV - 1);
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const float* base = p.partials + cb * a.HKV * R;
    for (int r = threadIdx.x; r < R; r += kAttnThreads) {
        float v = 0.f;
        for (int h = 0; h < a.HKV; ++h) v += __ldcg(base + int64_t(h) * R + r);
        const int64_t n = int64_t(c) * R + r;
        v += r == r_first ? res_first : __bfloat162float(p.res[int64_t(b) * p.ldr + n]);
        p.out[int64_t(b) * p.ldo + n] = __float2bfloat16_rn(v);
    }
    if (threadIdx.x == 0) atomicExch(p.counters + cb, 0u);
}

int attn_splits(const bq_attn_desc* d, int sm_count) {
    // enough CTAs to cover the SMs, each over >= 32 positions of the cache
    const int items = d->B * d->HKV;
    int sp = (2 * sm_count + items - 1) / items;
    sp = std::min(sp, std::max(1, d->S / 32));
    return std::max(1, std::min(sp, 32));
}

int validate_attn(const bq_attn_desc* d) {
    if (!d) return set_error(BQ_ERR_INVALID_ARG, "desc is NULL");
    if (d->B < 1 || d->HQ < 1 || d->HKV < 1 || d->S < 1)
        return set_error(BQ_ERR_SHAPE, "B, HQ, HKV, S must be positive");
    if (d->D != 64 && d->D != 128) return set_error(BQ_ERR_SHAPE, "head dim %d not supported (64 or 128)", d->D);
    if (int64_t(d->B) * d->HKV > kAttnMaxPairs)
        return set_error(BQ_ERR_SHAPE, "B * HKV = %lld exceeds %d", (long long)d->B * d->HKV, kAttnMaxPairs);
    if (d->HQ % d->HKV || d->HQ / d->HKV > kMaxG)
        return set_error(BQ_ERR_SHAPE, "HQ=%d must be a multiple of HKV=%d, at most %d query heads per kv head", d->HQ,
                         d->HKV, kMaxG);
    if (!d->qkv || !d->cos || !d->sin || !d->pos || !d->k_cache || !d->v_cache || !d->out)
        return set_error(BQ_ERR_INVALID_ARG, "qkv, cos, sin, pos, caches and out must be non-NULL");
    if ((d->q_norm == nullptr) != (d->k_norm == nullptr))
        return set_error(BQ_ERR_INVALID_ARG, "q_norm and k_norm must be given together");
    if (d->mask && d->mask_dtype != BQ_DT_BF16 && d->mask_dtype != BQ_DT_F32)
        return set_error(BQ_ERR_INVALID_ARG, "mask must be bf16 or f32 (additive)");
    const int vec = d->D / 32 * 2;  // bytes per lane of a row
    if ((reinterpret_cast<uintptr_t>(d->k_cache) | reinterpret_cast<uintptr_t>(d->v_cache)) % vec)
        return set_error(BQ_ERR_ALIGN, "caches must be %d-byte aligned", vec);
    if (d->ldqkv < int64_t(d->HQ + 2 * d->HKV) * d->D) return set_error(BQ_ERR_SHAPE, "ldqkv too small");
    if (d->ldo < int64_t(d->HQ) * d->D) return set_error(BQ_ERR_SHAPE, "ldo too small");
    return BQ_OK;
}


// Output rows per CTA of the fused attention + O projection: a multiple of 16
// dividing N, at most 64, and the Wo slice (R x G D bf16) within 48 KB.
int attn_o_rows(const bq_attn_o_desc* d) {
    const int GD = d->attn.HQ / d->attn.HKV * d->attn.D;
    for (int r = 64; r >= 16; r /= 2)
        if (d->N % r == 0 && r * GD * 2 <= 48 * 1024) return r;
    return 0;
}

int validate_attn_o(const bq_attn_o_desc* d) {
    if (!d) return set_error(BQ_ERR_INVALID_ARG, "desc is NULL");
    bq_attn_desc ad = d->attn;
    ad.out = d->out;  // the attention output stays on chip; out / ldo are checked below
    ad.ldo = int64_t(d->attn.HQ) * d->attn.D;
    int rc = validate_attn(&ad);
    if (rc) return rc;
    if (d->attn.B > kAttnOMaxB) return set_error(BQ_ERR_SHAPE, "B=%d exceeds %d", d->attn.B, kAttnOMaxB);
    if (d->attn.S > kAttnOMaxS) return set_error(BQ_ERR_SHAPE, "cache length %d exceeds %d", d->attn.S, kAttnOMaxS);
    if (d->N < 16 || !attn_o_rows(d)) return set_error(BQ_ERR_SHAPE, "N=%d must be a positive multiple of 16", d->N);
    if (int64_t(d->N / attn_o_rows(d)) * d->attn.B > kAttnMaxPairs) return set_error(BQ_ERR_SHAPE, "N=%d too large", d->N);
    if (!d->wo || !d->residual || !d->out) return set_error(BQ_ERR_INVALID_ARG, "wo, residual and out must be non-NULL");
    const int64_t K = int64_t(d->attn.HQ) * d->attn.D;
    if (d->ldw < K || d->ldr < d->N || d->ldo < d->N) return set_error(BQ_ERR_SHAPE, "ldw, ldr or ldo too small");
    if ((reinterpret_cast<uintptr_t>(d->wo) & 15) || (d->ldw * 2) % 16)
        return set_error(BQ_ERR_ALIGN, "wo and its row stride must be 16-byte aligned");
    return BQ_OK;
}
}  // namespace

}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_attention_workspace_bytes(const bq_attn_desc* d, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    int rc = validate_attn(d);
    if (rc) return rc;
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    const int sp = attn_splits(d, dev->sm_count);
    const int G = d->HQ / d->HKV;
    const size_t counters = kAttnCounterBytes;
    *bytes = sp == 1 ? 0 : counters + size_t(d->B) * d->HKV * sp * G * (d->D + 2) * 4;
    return BQ_OK;
}

int32_t bq_attention_step(const bq_attn_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate_attn(d);
    if (rc) return rc;
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    AttnParams p;
    std::memset(&p, 0, sizeof(p));
    p.B = d->B;
    p.HQ = d->HQ;
    p.HKV = d->HKV;
    p.S = d->S;
    p.G = d->HQ / d->HKV;
    p.splits = attn_splits(d, dev->sm_count);
    p.mask_dtype = d->mask_dtype;
    p.has_norm = d->q_norm != nullptr;
    p.eps = d->eps;
    p.scale = 1.0f / sqrtf(float(d->D));
    p.qkv = static_cast<const __nv_bfloat16*>(d->qkv);
    p.ldqkv = d->ldqkv;
    p.cos = static_cast<const __nv_bfloat16*>(d->cos);
    p.sin = static_cast<const __nv_bfloat16*>(d->sin);
    p.ldcs = d->ldcs;
    p.pos = d->pos;
    p.kc = static_cast<__nv_bfloat16*>(d->k_cache);
    p.vc = static_cast<__nv_bfloat16*>(d->v_cache);
    p.mask = d->mask;
    p.ldm = d->ldm;
    p.qn = static_cast<const __nv_bfloat16*>(d->q_norm);
    p.kn = static_cast<const __nv_bfloat16*>(d->k_norm);
    p.out = static_cast<__nv_bfloat16*>(d->out);
    p.ldo = d->ldo;
    if (p.splits > 1) {
        const size_t counters = kAttnCounterBytes;
        const size_t need = counters + size_t(d->B) * d->HKV * p.splits * p.G * (d->D + 2) * 4;
        if (!workspace || workspace_bytes < need)
            return set_error(BQ_ERR_WORKSPACE, "attention workspace of %zu bytes given, %zu needed", workspace_bytes, need);
        if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
        p.counters = static_cast<unsigned int*>(workspace);
        p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + counters);
    }
    // the splits of a (row, kv head) as one cluster when they fit the portable size
    const bool cluster = p.splits > 1 && p.splits <= 8;
    const void* fn = d->D == 128 ? (cluster ? reinterpret_cast<const void*>(&attention_step_kernel<4, true>)
                                            : reinterpret_cast<const void*>(&attention_step_kernel<4, false>))
                                 : (cluster ? reinterpret_cast<const void*>(&attention_step_kernel<2, true>)
                                            : reinterpret_cast<const void*>(&attention_step_kernel<2, false>));
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(p.splits, d->HKV, d->B);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (d->flags & BQ_FLAG_PDL) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = unsigned(p.splits);
        attr[na].val.clusterDim.y = 1;
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = na ? attr : nullptr;
    cfg.numAttrs = na;
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "attention launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

int32_t bq_attention_o_workspace_bytes(const bq_attn_o_desc* d, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    const int rc = validate_attn_o(d);
    if (rc) return rc;
    const int R = attn_o_rows(d);
    *bytes = kAttnCounterBytes + size_t(d->N / R) * d->attn.HKV * d->attn.B * R * 4;
    return BQ_OK;
}

int32_t bq_attention_o_step(const bq_attn_o_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate_attn_o(d);
    if (rc) return rc;
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    const bq_attn_desc* ad = &d->attn;
    // 32-row chunks when the grid still fits two CTAs per SM: each CTA's Wo slice
    // and partial rows halve (depth frame at B = 1: 6156 -> 5947 us); beyond that
    // the CTAs run in waves (B = 2: 6392 -> 7030 us) and 64-row chunks stay
    int R = attn_o_rows(d);
    if (R > 32 && d->N % 32 == 0 && int64_t(d->N / 32) * ad->HKV * ad->B <= 2 * int64_t(dev->sm_count) &&
        int64_t(d->N / 32) * ad->B <= kAttnMaxPairs)
        R = 32;
    const int chunks = d->N / R;
    const size_t need = kAttnCounterBytes + size_t(chunks) * ad->HKV * ad->B * R * 4;
    if (!workspace || workspace_bytes < need)
        return set_error(BQ_ERR_WORKSPACE, "attention + O workspace of %zu bytes given, %zu needed", workspace_bytes, need);
    if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
    AttnOParams p;
    std::memset(&p, 0, sizeof(p));
    p.a.B = ad->B;
    p.a.HQ = ad->HQ;
    p.a.HKV = ad->HKV;
    p.a.S = ad->S;
    p.a.G = ad->HQ / ad->HKV;
    p.a.splits = 1;
    p.a.mask_dtype = ad->mask_dtype;
    p.a.has_norm = ad->q_norm != nullptr;
    p.a.eps = ad->eps;
    p.a.scale = 1.0f / sqrtf(float(ad->D));
    p.a.qkv = static_cast<const __nv_bfloat16*>(ad->qkv);
    p.a.ldqkv = ad->ldqkv;
    p.a.cos = static_cast<const __nv_bfloat16*>(ad->cos);
    p.a.sin = static_cast<const __nv_bfloat16*>(ad->sin);
    p.a.ldcs = ad->ldcs;
    p.a.pos = ad->pos;
    p.a.kc = static_cast<__nv_bfloat16*>(ad->k_cache);
    p.a.vc = static_cast<__nv_bfloat16*>(ad->v_cache);
    p.a.mask = ad->mask;
    p.a.ldm = ad->ldm;
    p.a.qn = static_cast<const __nv_bfloat16*>(ad->q_norm);
    p.a.kn = static_cast<const __nv_bfloat16*>(ad->k_norm);
    p.R = R;
    p.wo = static_cast<const __nv_bfloat16*>(d->wo);
    p.ldw = d->ldw;
    p.res = static_cast<const __nv_bfloat16*>(d->residual);
    p.ldr = d->ldr;
    p.out = static_cast<__nv_bfloat16*>(d->out);
    p.ldo = d->ldo;
    p.counters = static_cast<unsigned int*>(workspace);
    p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kAttnCounterBytes);
    // a cluster of the HKV head CTAs of each (chunk, row) when it fits the portable size
    const bool cluster = ad->HKV <= 8;
    const void* fn = ad->D == 128 ? (cluster ? reinterpret_cast<const void*>(&attention_o_kernel<4, true>)
                                             : reinterpret_cast<const void*>(&attention_o_kernel<4, false>))
                                  : (cluster ? reinterpret_cast<const void*>(&attention_o_kernel<2, true>)
                                             : reinterpret_cast<const void*>(&attention_o_kernel<2, false>));
    const uint32_t smem = uint32_t(R) * p.a.G * ad->D * 2 + uint32_t(p.a.G) * ad->D * 4;
    rc = ensure_smem_attr(fn, smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(chunks, ad->HKV, ad->B);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[2];
    int na = 0;
    if (ad->flags & BQ_FLAG_PDL) {
        attr[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[na].val.programmaticStreamSerializationAllowed = 1;
        ++na;
    }
    if (cluster) {
        attr[na].id = cudaLaunchAttributeClusterDimension;
        attr[na].val.clusterDim.x = 1;
        attr[na].val.clusterDim.y = unsigned(ad->HKV);
        attr[na].val.clusterDim.z = 1;
        ++na;
    }
    cfg.attrs = na ? attr : nullptr;
    cfg.numAttrs = na;
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "attention + O launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
