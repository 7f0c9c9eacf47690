// fp32 output heads for sm_100a (bq_head_gemv): out = y @ W with fp32 weights,
// where y is the input rows or their RMSNorm computed with the reference's
// bf16 roundings (models/breeze.py:115-120). Two weight layouts:
//   N-major [N, K] (the backbone lm_head.float(), backbone_graph.py:70,273):
//     one warp per output row, 16-byte loads along K, shuffle reduction;
//   K-major [K, N] (one BreezeCodebooksHead slice, breeze.py:598-613):
//     a CTA takes 128 consecutive columns and a slice of K (coalesced 512-byte
//     rows), the K slices are summed by the last CTA to finish the tile in a
//     fixed order (deterministic).
// Weights are static, so each CTA pulls its share into L2 before the
// dependent-launch wait; the input rows are read after it.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

namespace {

constexpr int kHeadThreads = 256;
constexpr int kHeadMaxM = 16;
constexpr int kKnCols = 128;  // K-major: columns per CTA
// Fixed counter region: the arrival counters of every call sit at the same
// bytes, which no call's partial sums ever touch (a shape-dependent region
// would let one call's partials land where a later, larger call counts).
constexpr int kKnMaxTiles = 1024;
constexpr size_t kKnCounterBytes = size_t(kKnMaxTiles) * 4;

struct HeadParams {
    int32_t M, N, K, x_dtype, has_norm, splits, tiles, vec;
    float eps;
    const void* x;
    int64_t ldx;
    const __nv_bfloat16* gamma;
    const float* w;
    int64_t ldw;
    float* out;
    int64_t ldo;
    unsigned int* counters;  // [tiles]
    float* partials;         // [splits][M][N]
};

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Input rows as fp32 in shared memory, y[m * K + k]. With gamma: the
// reference's BreezeRMSNorm, xh = bf16(x * rsqrt(mean(x^2) + eps)), then
// y = bf16(gamma * xh).
__device__ void stage_rows(const HeadParams& p, float* y) {
    __shared__ float s_inv[kHeadMaxM];
    for (int i = threadIdx.x; i < p.M * p.K; i += blockDim.x) {
        const int m = i / p.K, k = i - m * p.K;
        y[i] = load_act(p.x, int64_t(m) * p.ldx + k, p.x_dtype);
    }
    __syncthreads();
    if (!p.has_norm) return;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int m = warp; m < p.M; m += blockDim.x >> 5) {
        float ss = 0.f;
        for (int k = lane; k < p.K; k += 32) ss = fmaf(y[m * p.K + k], y[m * p.K + k], ss);
        ss = warp_sum(ss);
        if (lane == 0) s_inv[m] = rsqrtf(ss / float(p.K) + p.eps);
    }
    __syncthreads();
    for (int i = threadIdx.x; i < p.M * p.K; i += blockDim.x) {
        const int m = i / p.K, k = i - m * p.K;
        const float xh = __bfloat162float(__float2bfloat16_rn(y[i] * s_inv[m]));
        y[i] = __bfloat162float(__float2bfloat16_rn(__bfloat162float(p.gamma[k]) * xh));
    }
    __syncthreads();
}

// ---- N-major: rows [r0, r1) per CTA, warp w takes r0 + w, r0 + w + 8, ...
template <bool VEC>
__global__ void __launch_bounds__(kHeadThreads) head_nk_kernel(const HeadParams p) {
    extern __shared__ __align__(16) float y[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = int(int64_t(blockIdx.x) * p.N / gridDim.x), r1 = int(int64_t(blockIdx.x + 1) * p.N / gridDim.x);
    if (VEC && threadIdx.x == 0) {
        for (int n = r0; n < r1; ++n) {
            const char* row = reinterpret_cast<const char*>(p.w + int64_t(n) * p.ldw);
            for (int64_t off = 0; off < int64_t(p.K) * 4; off += 65536) {
                const int64_t left = int64_t(p.K) * 4 - off;
                asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(row + off),
                             "r"(uint32_t(left < 65536 ? left : 65536))
                             : "memory");
            }
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    stage_rows(p, y);
    for (int n = r0 + warp; n < r1; n += kHeadThreads / 32) {
        float acc[kHeadMaxM];
#pragma unroll
        for (int m = 0; m < kHeadMaxM; ++m) acc[m] = 0.f;
        const float* wr = p.w + int64_t(n) * p.ldw;
        if (VEC) {
#pragma unroll 4
            for (int k4 = lane; k4 < (p.K >> 2); k4 += 32) {
                const float4 w4 = __ldg(reinterpret_cast<const float4*>(wr) + k4);
#pragma unroll
                for (int m = 0; m < kHeadMaxM; ++m) {
                    if (m < p.M) {
                        const float4 y4 = *reinterpret_cast<const float4*>(y + m * p.K + 4 * k4);
                        acc[m] = fmaf(y4.x, w4.x, fmaf(y4.y, w4.y, fmaf(y4.z, w4.z, fmaf(y4.w, w4.w, acc[m]))));
                    }
                }
            }
        } else {
#pragma unroll 4
            for (int k = lane; k < p.K; k += 32) {
                const float wv = __ldg(wr + k);
#pragma unroll
                for (int m = 0; m < kHeadMaxM; ++m)
                    if (m < p.M) acc[m] = fmaf(y[m * p.K + k], wv, acc[m]);
            }
        }
#pragma unroll
        for (int m = 0; m < kHeadMaxM; ++m) {
            if (m < p.M) {
                const float v = warp_sum(acc[m]);
                if (lane == 0) p.out[int64_t(m) * p.ldo + n] = v;
            }
        }
    }
}

// ---- K-major: CTA (tile, split) = columns [128 tile, +128) x K slice split
__global__ void __launch_bounds__(kHeadThreads) head_kn_kernel(const HeadParams p) {
    extern __shared__ __align__(16) float y[];
    __shared__ float red[kHeadMaxM][kKnCols];
    __shared__ unsigned int s_last;
    const int tile = blockIdx.x, split = blockIdx.y;
    const int n0 = tile * kKnCols;
    const int k0 = int(int64_t(split) * p.K / p.splits), k1 = int(int64_t(split + 1) * p.K / p.splits);
    const int col = threadIdx.x & (kKnCols - 1), rg = threadIdx.x >> 7;
    const int n = n0 + col;
    const int ncols = min(kKnCols, p.N - n0);
    // this CTA's weight rows: 4 bytes x ncols from row k, one 128-byte line per prefetch
    {
        const int lines = (ncols * 4 + 127) / 128 + 1;
        for (int t = threadIdx.x; t < (k1 - k0) * lines; t += kHeadThreads) {
            const int k = k0 + t / lines, l = t - (t / lines) * lines;
            const char* a = reinterpret_cast<const char*>(p.w + int64_t(k) * p.ldw + n0) + l * 128;
            if (a < reinterpret_cast<const char*>(p.w + int64_t(k) * p.ldw + n0 + ncols))
                asm volatile("prefetch.global.L2 [%0];" ::"l"(a));
        }
    }
    pdl_launch_dependents();
    pdl_wait();
    stage_rows(p, y);
    float acc[kHeadMaxM];
#pragma unroll
    for (int m = 0; m < kHeadMaxM; ++m) acc[m] = 0.f;
    if (n < p.N) {
        const float* wc = p.w + n;
#pragma unroll 8
        for (int k = k0 + rg; k < k1; k += 2) {
            const float wv = __ldg(wc + int64_t(k) * p.ldw);
#pragma unroll
            for (int m = 0; m < kHeadMaxM; ++m)
                if (m < p.M) acc[m] = fmaf(y[m * p.K + k], wv, acc[m]);
        }
    }
    // the two row groups of the CTA
    if (rg == 1) {
#pragma unroll
        for (int m = 0; m < kHeadMaxM; ++m)
            if (m < p.M) red[m][col] = acc[m];
    }
    __syncthreads();
    if (rg == 0) {
#pragma unroll
        for (int m = 0; m < kHeadMaxM; ++m)
            if (m < p.M) acc[m] += red[m][col];
    }
    if (p.splits == 1) {
        if (rg == 0 && n < p.N) {
#pragma unroll
            for (int m = 0; m < kHeadMaxM; ++m)
                if (m < p.M) p.out[int64_t(m) * p.ldo + n] = acc[m];
        }
        return;
    }
    // split K: partials, then the last CTA of the tile sums them in split order
    if (rg == 0 && n < p.N) {
#pragma unroll
        for (int m = 0; m < kHeadMaxM; ++m)
            if (m < p.M) __stcg(p.partials + (int64_t(split) * p.M + m) * p.N + n, acc[m]);
    }
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) s_last = atomicAdd(p.counters + tile, 1u) == unsigned(p.splits - 1) ? 1u : 0u;
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    if (rg == 0 && n < p.N) {
        for (int m = 0; m < p.M; ++m) {
            float t = 0.f;
            for (int s = 0; s < p.splits; ++s) t += __ldcg(p.partials + (int64_t(s) * p.M + m) * p.N + n);
            p.out[int64_t(m) * p.ldo + n] = t;
        }
    }
    if (threadIdx.x == 0) atomicExch(p.counters + tile, 0u);
}

int validate_head(const bq_head_desc* d) {
    if (!d) return set_error(BQ_ERR_INVALID_ARG, "desc is NULL");
    if (d->M < 1 || d->M > kHeadMaxM || d->N < 1 || d->K < 1)
        return set_error(BQ_ERR_SHAPE, "head: M in [1, %d], N and K positive (got %d, %d, %d)", kHeadMaxM, d->M, d->N,
                         d->K);
    if (d->layout != BQ_HEAD_NK && d->layout != BQ_HEAD_KN) return set_error(BQ_ERR_INVALID_ARG, "unknown head layout %d", d->layout);
    if (d->x_dtype < BQ_DT_BF16 || d->x_dtype > BQ_DT_F32) return set_error(BQ_ERR_INVALID_ARG, "unknown dtype %d", d->x_dtype);
    if (!d->x || !d->w || !d->out) return set_error(BQ_ERR_INVALID_ARG, "x, w and out must be non-NULL");
    if (d->ldx < d->K || d->ldo < d->N) return set_error(BQ_ERR_SHAPE, "ldx < K or ldo < N");
    if (d->layout == BQ_HEAD_NK ? d->ldw < d->K : d->ldw < d->N) return set_error(BQ_ERR_SHAPE, "ldw too small");
    if (d->layout == BQ_HEAD_KN && (d->N + kKnCols - 1) / kKnCols > kKnMaxTiles)
        return set_error(BQ_ERR_SHAPE, "head: N=%d exceeds %d columns", d->N, kKnMaxTiles * kKnCols);
    if (size_t(d->M) * d->K * 4 > 96 * 1024)
        return set_error(BQ_ERR_SHAPE, "head: M * K = %d inputs do not fit in shared memory", d->M * d->K);
    return BQ_OK;
}

void kn_grid(const bq_head_desc* d, int sm_count, int* tiles, int* splits) {
    *tiles = (d->N + kKnCols - 1) / kKnCols;
    int s = (2 * sm_count + *tiles - 1) / *tiles;
    s = std::min(s, std::max(1, d->K / 16));
    *splits = std::max(1, std::min(s, 64));
}



}  // namespace
}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_head_workspace_bytes(const bq_head_desc* d, size_t* bytes) {
    if (!bytes) return set_error(BQ_ERR_INVALID_ARG, "bytes is NULL");
    int rc = validate_head(d);
    if (rc) return rc;
    *bytes = 0;
    if (d->layout == BQ_HEAD_KN) {
        const DeviceInfo* dev = device_info();
        if (!dev) return BQ_ERR_CUDA;
        int tiles, splits;
        kn_grid(d, dev->sm_count, &tiles, &splits);
        if (splits > 1) *bytes = kKnCounterBytes + size_t(splits) * d->M * d->N * 4;
    }
    return BQ_OK;
}

int32_t bq_head_gemv(const bq_head_desc* d, void* workspace, size_t workspace_bytes, void* stream) {
    int rc = validate_head(d);
    if (rc) return rc;
    const DeviceInfo* dev = device_info();
    if (!dev) return BQ_ERR_CUDA;
    if (dev->major != 10) return set_error(BQ_ERR_DEVICE, "sm_%d%d device: this library is built for sm_100a", dev->major, dev->minor);
    HeadParams p;
    std::memset(&p, 0, sizeof(p));
    p.M = d->M;
    p.N = d->N;
    p.K = d->K;
    p.x_dtype = d->x_dtype;
    p.has_norm = d->gamma != nullptr;
    p.eps = d->eps;
    p.x = d->x;
    p.ldx = d->ldx;
    p.gamma = static_cast<const __nv_bfloat16*>(d->gamma);
    p.w = d->w;
    p.ldw = d->ldw;
    p.out = d->out;
    p.ldo = d->ldo;
    const uint32_t smem = uint32_t(d->M) * d->K * 4;
    const void* fn;
    dim3 grid;
    if (d->layout == BQ_HEAD_NK) {
        p.vec = (reinterpret_cast<uintptr_t>(d->w) % 16 == 0 && d->ldw % 4 == 0 && d->K % 4 == 0) ? 1 : 0;
        fn = p.vec ? reinterpret_cast<const void*>(&head_nk_kernel<true>) : reinterpret_cast<const void*>(&head_nk_kernel<false>);
        grid = dim3(std::max(1, std::min((d->N + 7) / 8, 2 * dev->sm_count)));
    } else {
        kn_grid(d, dev->sm_count, &p.tiles, &p.splits);
        if (p.splits > 1) {
            const size_t cb = kKnCounterBytes;
            const size_t need = cb + size_t(p.splits) * d->M * d->N * 4;
            if (!workspace || workspace_bytes < need)
                return set_error(BQ_ERR_WORKSPACE, "head workspace of %zu bytes given, %zu needed", workspace_bytes, need);
            if (reinterpret_cast<uintptr_t>(workspace) & 255) return set_error(BQ_ERR_ALIGN, "workspace must be 256-byte aligned");
            p.counters = static_cast<unsigned int*>(workspace);
            p.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + cb);
        }
        fn = reinterpret_cast<const void*>(&head_kn_kernel);
        grid = dim3(p.tiles, p.splits);
    }
    rc = ensure_smem_attr(fn, smem);
    if (rc) return rc;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = grid;
    cfg.blockDim = dim3(kHeadThreads);
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
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "head launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
