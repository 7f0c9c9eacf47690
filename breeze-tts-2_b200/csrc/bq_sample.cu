// CFG mix and token sampling for sm_100a (bq_sample): one CTA (512 or 1024
// threads, by vocabulary size) per sample row. The row's logits are mixed (cond/uncond), masked and
// penalised in registers, sorted once (CUB block radix sort, descending), and
// top-k, top-p, the softmax and the inverse-CDF draw all work on the sorted
// order with block scans. Follows DepthDecoderGraph._cfg_sample
// (models/cudagraph/depth_decoder_graph.py:487-558) and sample_logits
// (models/cudagraph/sampling.py:36-87): temperature -> top_k -> top_p on raw
// logits -> softmax -> one draw; greedy = argmax of the mixed, masked logits.
//
// Random numbers: Philox4x32-10 (Salmon, Moraes, Dror and Shaw, "Parallel
// random numbers: as easy as 1, 2, 3", SC 2011), key = rng[0], counter =
// {rng[1] low, rng[1] high, row, 0}; u = (first word >> 8) * 2^-24. The last
// CTA to finish advances rng[1], so each launch (and each graph replay) draws
// new numbers without a host round trip.
#include <cub/block/block_radix_sort.cuh>
#include <cub/block/block_scan.cuh>
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cstring>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

namespace {


struct SampleParams {
    int32_t rows, V, cfg, max_k, mask_lo, mask_hi, clamp_hi, topk_value, history_cap, flags_off, append;
    float rep_penalty;
    const float* logits;
    int64_t ldl;
    const float* guidance;
    const float* temperature;
    const int64_t* top_k;
    const float* top_p;
    const int64_t* do_sample;
    int64_t* history;
    int32_t* history_len;
    const uint8_t* suppress;
    const float* uniform;
    unsigned long long* rng;
    float* cfg_out;
    int64_t ldc;
    int64_t* tokens;
    int64_t ldt;
    int64_t* tokens2;
    int64_t ldt2;
    long long eos_id;
    int32_t* eos_flag;
    unsigned int* arrive;
};

constexpr int kFastK = 128;  // top-k up to this size skips the full sort

// Order-preserving unsigned image of a float (larger float -> larger key).
__device__ __forceinline__ uint32_t ordered_bits(float f) {
    const uint32_t b = __float_as_uint(f);
    return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ uint4 philox4x32_10(uint4 c, uint2 k) {
#pragma unroll
    for (int i = 0; i < 10; ++i) {
        const uint32_t hi0 = __umulhi(0xD2511F53u, c.x), lo0 = 0xD2511F53u * c.x;
        const uint32_t hi1 = __umulhi(0xCD9E8D57u, c.z), lo1 = 0xCD9E8D57u * c.z;
        c = make_uint4(hi1 ^ c.y ^ k.x, lo1, hi0 ^ c.w ^ k.y, lo0);
        k.x += 0x9E3779B9u;
        k.y += 0xBB67AE85u;
    }
    return c;
}

// Block-wide helpers over THREADS threads (scratch: THREADS / 32 entries).
template <int THREADS, bool MAX>
__device__ __forceinline__ int block_reduce_int(int v, int* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const int w = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? max(v, w) : min(v, w);
    }
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    v = lane < THREADS / 32 ? scratch[lane] : (MAX ? INT_MIN : INT_MAX);
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const int w = __shfl_xor_sync(0xffffffffu, v, o);
        v = MAX ? max(v, w) : min(v, w);
    }
    __syncthreads();
    return v;
}
// (value, index) argmax: largest value, smallest index among equal values.
template <int THREADS>
__device__ __forceinline__ int block_argmax(float v, int i, float* sv, int* si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
        }
    }
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = i;
    }
    __syncthreads();
    v = lane < THREADS / 32 ? sv[lane] : -INFINITY;
    i = lane < THREADS / 32 ? si[lane] : INT_MAX;
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (ov > v || (ov == v && oi < i)) {
            v = ov;
            i = oi;
        }
    }
    __syncthreads();
    return i;
}

template <int THREADS, int ITEMS>
struct SampleTypes {
    using Sort = cub::BlockRadixSort<float, THREADS, ITEMS, int>;
    using Scan = cub::BlockScan<float, THREADS>;
    union Temp {
        typename Sort::TempStorage sort;
        typename Scan::TempStorage scan;
    };
};

template <int THREADS, int ITEMS>
__global__ void __launch_bounds__(THREADS) sample_kernel(const SampleParams p) {
    using T = SampleTypes<THREADS, ITEMS>;
    extern __shared__ __align__(16) unsigned char smem[];
    auto& temp = *reinterpret_cast<typename T::Temp*>(smem);
    uint8_t* hflag = smem + p.flags_off;  // [V] repetition-penalty flags
    __shared__ float s_f[32];
    __shared__ int s_i[32];
    __shared__ int s_tok;
    __shared__ unsigned int s_last;
    __shared__ unsigned int s_hist[256];
    __shared__ int s_sel[4];
    __shared__ float s_ck[kFastK], s_sk[kFastK];
    __shared__ int s_ci[kFastK], s_si[kFastK];
    const int r = blockIdx.x, t = threadIdx.x;

    unsigned long long calls = 0, seed = 0;
    if (!p.uniform) {
        seed = p.rng[0];
        calls = p.rng[1];
    }
    pdl_launch_dependents();
    pdl_wait();  // logits (and the parameter buffers) come from earlier kernels

    if (p.history && p.append && t == 0) {
        // the row's current token (the previous step's draw) joins its history
        const int n = p.history_len[r];
        if (n < p.history_cap) {
            p.history[int64_t(r) * p.history_cap + n] = p.tokens[int64_t(r) * p.ldt];
            p.history_len[r] = n + 1;
        }
    }
    __syncthreads();
    const bool pen = p.history != nullptr && p.rep_penalty != 1.f;
    if (pen) {
        for (int v = t; v < p.V; v += THREADS) hflag[v] = 0;
        __syncthreads();
        const int n = min(p.history_len[r], p.history_cap);
        for (int i = t; i < n; i += THREADS) {
            const int64_t h = p.history[int64_t(r) * p.history_cap + i];
            if (h >= 0 && h < p.V) hflag[h] = 1;
        }
        __syncthreads();
    }

    // ---- mixed, masked logits (blocked: thread t holds [t * ITEMS, +ITEMS))
    const float* cond = p.logits + int64_t(r) * p.ldl;
    const float* unc = p.cfg ? p.logits + int64_t(r + p.rows) * p.ldl : nullptr;
    const float g = p.cfg ? p.guidance[r] : 0.f;
    const float temp_r = p.temperature[r];
    float key[ITEMS];
    int idx[ITEMS];
    float gv = -INFINITY;
    int gi = INT_MAX;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const int v = t * ITEMS + j;
        if (v < p.V) {
            float c = cond[v];
            if (p.cfg) {
                const float u = unc[v];
                c = __fadd_rn(u, __fmul_rn(g, __fsub_rn(c, u)));  // uncond + g * (cond - uncond)
            }
            if (v >= p.mask_lo && v < p.mask_hi) c = -INFINITY;
            if (pen && hflag[v]) c = c > 0.f ? __fdiv_rn(c, p.rep_penalty) : __fmul_rn(c, p.rep_penalty);
            if (p.suppress && p.suppress[v]) c = -INFINITY;
            if (p.cfg_out) p.cfg_out[int64_t(r) * p.ldc + v] = c;
            if (c > gv || (c == gv && v < gi)) {
                gv = c;
                gi = v;
            }
            key[j] = __fdiv_rn(c, temp_r);
            idx[j] = v;
        } else {
            key[j] = -INFINITY;
            idx[j] = INT_MAX;
        }
    }
    const int greedy = block_argmax<THREADS>(gv, gi, s_f, s_i);

    int k = int(p.top_k[r]);
    if (k <= 0) k = p.max_k;
    k = max(1, min(k, min(p.max_k, p.V)));
    float u;
    if (p.uniform) {
        u = p.uniform[r];
    } else {
        const uint4 c = philox4x32_10(make_uint4(uint32_t(calls), uint32_t(calls >> 32), uint32_t(r), 0u),
                                      make_uint2(uint32_t(seed), uint32_t(seed >> 32)));
        u = float(c.x >> 8) * (1.0f / 16777216.0f);
    }
    const float tp = p.top_p[r];
    int sel = INT_MIN;  // rank of the drawn token among the kept ones (INT_MIN: nothing kept)
    bool done = false;

    // ---- fast path (k <= kFastK): radix-select the k-th largest scaled logit
    // (4 passes of 8 bits over order-preserving keys), keep the candidates
    // (ties at the threshold by ascending index for rank-based top-k), rank
    // them by counting and finish top-p, softmax and the draw in one warp.
    if (k <= kFastK) {
        uint32_t uk[ITEMS];
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) uk[j] = ordered_bits(key[j]);
        uint32_t prefix = 0, pmask = 0;
        int rem = k;
#pragma unroll 1
        for (int pass = 0; pass < 4; ++pass) {
            const int shift = 24 - 8 * pass;
            for (int i = t; i < 256; i += THREADS) s_hist[i] = 0;
            __syncthreads();
#pragma unroll
            for (int j = 0; j < ITEMS; ++j)
                if ((uk[j] & pmask) == prefix) atomicAdd(&s_hist[(uk[j] >> shift) & 255u], 1u);
            __syncthreads();
            if (t < 32) {
                // lane l owns bins 255 - 8l - q (q = 0..7), largest digits first
                int c[8], sum = 0;
#pragma unroll
                for (int q = 0; q < 8; ++q) {
                    c[q] = int(s_hist[255 - 8 * t - q]);
                    sum += c[q];
                }
                int incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const int v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (t >= o) incl += v;
                }
                const int excl = incl - sum;
                if (excl < rem && rem <= incl) {
                    int acc = excl;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        if (acc + c[q] >= rem) {
                            s_sel[0] = 255 - 8 * t - q;
                            s_sel[1] = acc;
                            break;
                        }
                        acc += c[q];
                    }
                }
            }
            __syncthreads();
            prefix |= uint32_t(s_sel[0]) << shift;
            pmask |= 0xFFu << shift;
            rem -= s_sel[1];
            __syncthreads();
        }
        // candidates: above the threshold, plus ties at it (the first `rem` by index for rank-based top-k)
        float tf[ITEMS], tr[ITEMS], tot;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) tf[j] = uk[j] == prefix ? 1.f : 0.f;
        typename T::Scan(temp.scan).ExclusiveSum(tf, tr, tot);
        __syncthreads();
        float take[ITEMS], pos[ITEMS], nc_f;
#pragma unroll
        for (int j = 0; j < ITEMS; ++j) {
            const bool tk = key[j] > -INFINITY &&
                            (uk[j] > prefix || (uk[j] == prefix && (p.topk_value || tr[j] < float(rem))));
            take[j] = tk ? 1.f : 0.f;
        }
        typename T::Scan(temp.scan).ExclusiveSum(take, pos, nc_f);
        __syncthreads();
        const int nc = int(nc_f);
        if (nc <= kFastK) {
#pragma unroll
            for (int j = 0; j < ITEMS; ++j) {
                if (take[j] > 0.f) {
                    s_ck[int(pos[j])] = key[j];
                    s_ci[int(pos[j])] = idx[j];
                }
            }
            __syncthreads();
            for (int c = t; c < nc; c += THREADS) {
                const float kc = s_ck[c];
                const int ic = s_ci[c];
                int rk = 0;
                for (int i = 0; i < nc; ++i) rk += (s_ck[i] > kc || (s_ck[i] == kc && s_ci[i] < ic)) ? 1 : 0;
                s_sk[rk] = kc;
                s_si[rk] = ic;
            }
            __syncthreads();
            if (t < 32) {
                // lane l holds ranks 4l .. 4l + 3
                const float mx = nc > 0 ? s_sk[0] : 0.f;
                float e[4], sum = 0.f;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int rk = 4 * t + q;
                    e[q] = rk < nc ? expf(s_sk[rk] - mx) : 0.f;
                    sum += e[q];
                }
                float incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (t >= o) incl += v;
                }
                const float z = __shfl_sync(0xffffffffu, incl, 31);
                float ex = incl - sum;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int rk = 4 * t + q;
                    if (rk >= 1 && ex / z > tp) e[q] = 0.f;  // mass before this rank exceeds top_p
                    ex += rk < nc ? expf(s_sk[rk] - mx) : 0.f;
                }
                sum = e[0] + e[1] + e[2] + e[3];
                incl = sum;
#pragma unroll
                for (int o = 1; o < 32; o <<= 1) {
                    const float v = __shfl_up_sync(0xffffffffu, incl, o);
                    if (t >= o) incl += v;
                }
                const float z2 = __shfl_sync(0xffffffffu, incl, 31);
                const float target = u * z2;
                float cum = incl - sum;
                int first = INT_MAX, last = INT_MIN;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    cum += e[q];
                    if (e[q] > 0.f) {
                        if (first == INT_MAX && cum > target) first = 4 * t + q;
                        last = 4 * t + q;
                    }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    first = min(first, __shfl_xor_sync(0xffffffffu, first, o));
                    last = max(last, __shfl_xor_sync(0xffffffffu, last, o));
                }
                if (t == 0) {
                    const int sl = first != INT_MAX ? first : last;
                    s_sel[2] = sl;
                    if (sl != INT_MIN) s_tok = s_si[sl];
                }
            }
            __syncthreads();
            sel = s_sel[2];
            done = true;
        }
    }

    if (!done) {
    // ---- sort descending; thread t then holds ranks [t * ITEMS, +ITEMS)
    typename T::Sort(temp.sort).SortDescending(key, idx);
    __syncthreads();
    if (t == 0) s_f[0] = key[0];
    if (t == (k - 1) / ITEMS) {
#pragma unroll
        for (int j = 0; j < ITEMS; ++j)
            if (j == (k - 1) % ITEMS) s_f[1] = key[j];
    }
    __syncthreads();
    const float mx = s_f[0], kth = s_f[1];
    float e[ITEMS];
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const int rank = t * ITEMS + j;
        const bool kept = (p.topk_value ? key[j] >= kth : rank < k) && key[j] > -INFINITY;
        e[j] = kept ? expf(key[j] - mx) : 0.f;
    }
    // top-p: drop rank i >= 1 when the probability mass before it exceeds top_p
    float excl[ITEMS], z;
    typename T::Scan(temp.scan).ExclusiveSum(e, excl, z);
    __syncthreads();
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const int rank = t * ITEMS + j;
        if (rank >= 1 && excl[j] / z > tp) e[j] = 0.f;
    }
    float cum[ITEMS], z2;
    typename T::Scan(temp.scan).InclusiveSum(e, cum, z2);
    __syncthreads();

    // ---- one draw: the first kept rank whose cumulative mass exceeds u * z2
    const float target = u * z2;
    int first = INT_MAX, last = INT_MIN;
#pragma unroll
    for (int j = 0; j < ITEMS; ++j) {
        const int rank = t * ITEMS + j;
        if (e[j] > 0.f) {
            if (first == INT_MAX && cum[j] > target) first = rank;
            last = rank;
        }
    }
    first = block_reduce_int<THREADS, false>(first, s_i);
    last = block_reduce_int<THREADS, true>(last, s_i);
    sel = first != INT_MAX ? first : last;  // u * z2 rounding up to z2 takes the last kept rank
    if (sel != INT_MIN && t == sel / ITEMS) {
#pragma unroll
        for (int j = 0; j < ITEMS; ++j)
            if (j == sel % ITEMS) s_tok = idx[j];
    }
    }
    __syncthreads();
    if (t == 0) {
        const bool sample = p.do_sample[r] != 0 && sel != INT_MIN;
        long long tok = sample ? s_tok : greedy;
        if (tok == INT_MAX) tok = 0;  // every logit was masked
        tok = tok < 0 ? 0 : (tok > p.clamp_hi ? p.clamp_hi : tok);
        p.tokens[int64_t(r) * p.ldt] = tok;
        if (p.cfg) p.tokens[int64_t(r + p.rows) * p.ldt] = tok;
        if (p.tokens2) {
            p.tokens2[int64_t(r) * p.ldt2] = tok;
            if (p.cfg) p.tokens2[int64_t(r + p.rows) * p.ldt2] = tok;
        }
        if (p.eos_flag && tok == p.eos_id) *p.eos_flag = 1;
        if (!p.uniform) {
            // the last CTA advances the call counter (every CTA has read it by now)
            __threadfence();
            s_last = atomicAdd(p.arrive, 1u) == unsigned(p.rows - 1) ? 1u : 0u;
            if (s_last) {
                p.rng[1] = calls + 1;
                atomicExch(p.arrive, 0u);
            }
        }
    }
}

template <int THREADS, int ITEMS>
size_t sample_temp_bytes() {
    return (sizeof(typename SampleTypes<THREADS, ITEMS>::Temp) + 15) / 16 * 16;
}

int validate_sample(const bq_sample_desc* d) {
    if (!d) return set_error(BQ_ERR_INVALID_ARG, "desc is NULL");
    if (d->rows < 1 || d->V < 1 || d->V > BQ_SAMPLE_MAX_V)
        return set_error(BQ_ERR_SHAPE, "sample: rows >= 1 and 1 <= V <= %d (got %d, %d)", BQ_SAMPLE_MAX_V, d->rows, d->V);
    if (d->max_k < 1) return set_error(BQ_ERR_SHAPE, "sample: max_k must be >= 1");
    if (d->mask_lo < 0 || d->mask_hi < d->mask_lo || d->mask_hi > d->V)
        return set_error(BQ_ERR_SHAPE, "sample: mask range [%d, %d) outside [0, %d]", d->mask_lo, d->mask_hi, d->V);
    if (!d->logits || !d->temperature || !d->top_k || !d->top_p || !d->do_sample || !d->tokens)
        return set_error(BQ_ERR_INVALID_ARG, "logits, temperature, top_k, top_p, do_sample and tokens must be non-NULL");
    if (d->cfg && !d->guidance) return set_error(BQ_ERR_INVALID_ARG, "cfg needs the guidance buffer");
    if (!d->uniform && !d->rng) return set_error(BQ_ERR_INVALID_ARG, "either uniform or rng must be given");
    if (d->history && (!d->history_len || d->history_cap < 1))
        return set_error(BQ_ERR_INVALID_ARG, "history needs history_len and history_cap >= 1");
    if (d->ldl < d->V || (d->cfg_out && d->ldc < d->V)) return set_error(BQ_ERR_SHAPE, "row stride smaller than V");
    if (d->rep_penalty <= 0.f) return set_error(BQ_ERR_INVALID_ARG, "repetition penalty must be > 0");
    return BQ_OK;
}

}  // namespace
}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_sample_workspace_bytes(const bq_sample_desc* d, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    int rc = validate_sample(d);
    if (rc) return rc;
    *bytes = 256;
    return BQ_OK;
}

int32_t bq_sample(const bq_sample_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate_sample(d);
    if (rc) return rc;
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    if (!d->uniform) {
        if (!workspace || workspace_bytes < 256) return set_error(BQ_ERR_WORKSPACE, "sample workspace of 256 bytes needed");
        if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
    }
    SampleParams p;
    std::memset(&p, 0, sizeof(p));
    p.rows = d->rows;
    p.V = d->V;
    p.cfg = d->cfg ? 1 : 0;
    p.max_k = d->max_k;
    p.mask_lo = d->mask_lo;
    p.mask_hi = d->mask_hi;
    p.clamp_hi = d->clamp_hi;
    p.topk_value = (d->flags & BQ_SAMPLE_TOPK_VALUE) ? 1 : 0;
    p.history_cap = d->history_cap;
    p.rep_penalty = d->rep_penalty;
    p.logits = d->logits;
    p.ldl = d->ldl;
    p.guidance = d->guidance;
    p.temperature = d->temperature;
    p.top_k = d->top_k;
    p.top_p = d->top_p;
    p.do_sample = d->do_sample;
    p.history = d->history;
    p.history_len = d->history_len;
    p.suppress = d->suppress;
    p.uniform = d->uniform;
    p.rng = reinterpret_cast<unsigned long long*>(d->rng);
    p.cfg_out = d->cfg_out;
    p.ldc = d->ldc;
    p.tokens = d->tokens;
    p.ldt = d->ldt;
    p.tokens2 = d->tokens2;
    p.ldt2 = d->ldt2;
    p.append = (d->flags & BQ_SAMPLE_APPEND_HISTORY) ? 1 : 0;
    p.eos_id = d->eos_id;
    p.eos_flag = d->eos_flag;
    p.arrive = static_cast<unsigned int*>(workspace);
    // V <= 2048: 512 threads x 4 keys; <= 4096: 512 x 8 (1024 x 4 measured slower); <= 8192: 1024 x 8
    const void* fn;
    size_t temp;
    int threads;
    if (d->V <= 2048) {
        fn = reinterpret_cast<const void*>(&sample_kernel<512, 4>);
        temp = sample_temp_bytes<512, 4>();
        threads = 512;
    } else if (d->V <= 4096) {
        fn = reinterpret_cast<const void*>(&sample_kernel<512, 8>);
        temp = sample_temp_bytes<512, 8>();
        threads = 512;
    } else {
        fn = reinterpret_cast<const void*>(&sample_kernel<1024, 8>);
        temp = sample_temp_bytes<1024, 8>();
        threads = 1024;
    }
    p.flags_off = int(temp);
    const uint32_t smem = uint32_t(temp + (size_t(d->V) + 15) / 16 * 16);
    rc = ensure_smem_attr(fn, smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(d->rows);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    if (d->flags & BQ_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    void* args[] = {&p};
    cudaError_t e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "sample launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
