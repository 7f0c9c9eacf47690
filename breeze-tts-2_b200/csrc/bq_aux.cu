// Layout, dequantization and glue kernels:
//   * tinygemm int4 re-tiling (replaces torch._convert_weight_to_int4pack,
//     models/int4_linear.py:59) and its inverse;
//   * fp32 dequantization of every weight format, bit-exact with the
//     reference's dequant (parity checks and debugging);
//   * RMSNorm and SiLU*up glue (models/fused/kernels.py:541-575).
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstring>

#include "bq_device.cuh"
#include "bq_host.h"

namespace bq {

// One thread per output int32 word of the tinygemm tensor
// [N/8, K/(16*ikt), 32, ikt/2]. Word (nt, ko, lane, j) serves row
// n = 8*nt + lane/4 and takes bytes B_i = 8*(ko*ikt + 2j) + lane%4 + 4i of
// that row: high nibbles (even k) go to nibbles 0..3, low nibbles (odd k) to
// nibbles 4..7, so each 16-bit lane pair is one {k, k+1} MMA operand pair.
__global__ void tinygemm_pack_kernel(const uint8_t* __restrict__ in, uint32_t* __restrict__ out, int N, int K,
                                     int ikt) {
    const int64_t words = int64_t(N / 8) * (K / (16 * ikt)) * 32 * (ikt / 2);
    const int half = ikt / 2, KO = K / (16 * ikt);
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < words;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int j = int(idx % half);
        const int lane = int((idx / half) % 32);
        const int ko = int((idx / (half * 32)) % KO);
        const int nt = int(idx / (int64_t(half) * 32 * KO));
        const int n = nt * 8 + lane / 4;
        const uint8_t* row = in + int64_t(n) * (K / 2);
        const int b0 = (ko * ikt + 2 * j) * 8 + (lane & 3);
        uint32_t w = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t v = row[b0 + 4 * i];
            w |= (v >> 4) << (4 * i);
            w |= (v & 15u) << (16 + 4 * i);
        }
        out[idx] = w;
    }
}

__global__ void tinygemm_unpack_kernel(const uint32_t* __restrict__ in, uint8_t* __restrict__ out, int N, int K,
                                       int ikt) {
    const int64_t words = int64_t(N / 8) * (K / (16 * ikt)) * 32 * (ikt / 2);
    const int half = ikt / 2, KO = K / (16 * ikt);
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < words;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int j = int(idx % half);
        const int lane = int((idx / half) % 32);
        const int ko = int((idx / (half * 32)) % KO);
        const int nt = int(idx / (int64_t(half) * 32 * KO));
        const int n = nt * 8 + lane / 4;
        uint8_t* row = out + int64_t(n) * (K / 2);
        const int b0 = (ko * ikt + 2 * j) * 8 + (lane & 3);
        const uint32_t w = in[idx];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t hi = (w >> (4 * i)) & 15u, lo = (w >> (16 + 4 * i)) & 15u;
            row[b0 + 4 * i] = uint8_t((hi << 4) | lo);
        }
    }
}

// W[n, k] in fp32, bit-exact with the reference's dequantization.
__global__ void dequant_kernel(bq_gemv_desc d, float* __restrict__ out) {
    const int64_t total = int64_t(d.N) * d.K;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int n = int(idx / d.K), k = int(idx % d.K);
        float v = 0.f;
        if (d.wfmt == BQ_W_INT4_TINYGEMM) {
            const int KO = d.K / 128, kr = k & 127, jj = kr >> 5, kl = kr & 31;
            const int lane = 4 * (n & 7) + ((kl & 7) >> 1);
            const int pos = 4 * (kl & 1) + (kl >> 3);
            const uint32_t w = static_cast<const uint32_t*>(d.w)[((int64_t(n >> 3) * KO + (k >> 7)) * 32 + lane) * 4 + jj];
            const int q = int((w >> (4 * pos)) & 15u);
            const __nv_bfloat16* sz = static_cast<const __nv_bfloat16*>(d.scale) + (int64_t(k / d.group) * d.N + n) * 2;
            v = __fmaf_rn(float(q - 8), __bfloat162float(sz[0]), __bfloat162float(sz[1]));
        } else if (d.wfmt == BQ_W_INT4_PLAIN) {
            const uint8_t b = static_cast<const uint8_t*>(d.w)[int64_t(n) * (d.K / 2) + (k >> 1)];
            const int q = (k & 1) ? (b >> 4) : (b & 15);
            const __nv_bfloat16* sz = static_cast<const __nv_bfloat16*>(d.scale) + (int64_t(k / 128) * d.N + n) * 2;
            v = __fmaf_rn(float(q), __bfloat162float(sz[0]), __bfloat162float(sz[1]));
        } else if (d.wfmt == BQ_W_FP8_E4M3) {
            const uint8_t b = static_cast<const uint8_t*>(d.w)[idx];
            const uint32_t h2 = e4m3x2_to_f16x2(uint16_t(b));
            const float q = __half2float(__ushort_as_half(uint16_t(h2 & 0xFFFF)));
            v = __fmul_rn(q, static_cast<const float*>(d.scale)[n]);
        } else if (d.wfmt == BQ_W_INT8) {
            const int8_t q = static_cast<const int8_t*>(d.w)[idx];
            const float s = __bfloat162float(__float2bfloat16_rn(static_cast<const float*>(d.scale)[n]));
            v = __bfloat162float(__float2bfloat16_rn(__fmul_rn(float(q), s)));
        } else {
            v = __bfloat162float(static_cast<const __nv_bfloat16*>(d.w)[idx]);
        }
        out[idx] = v;
    }
}

// One block per row: out = x * (1/sqrt(mean(x^2) + eps)) * gamma, fp32 math.
__global__ void rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, int64_t ldx, const __nv_bfloat16* __restrict__ g,
                               __nv_bfloat16* __restrict__ out, int64_t ldo, int K, float eps) {
    __shared__ float red[32];
    const __nv_bfloat16* xr = x + blockIdx.x * ldx;
    float ss = 0.f;
    for (int k = threadIdx.x; k < K; k += blockDim.x) {
        const float v = __bfloat162float(xr[k]);
        ss = fmaf(v, v, ss);
    }
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
        ss = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
        for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        if (threadIdx.x == 0) red[0] = 1.0f / sqrtf(ss / float(K) + eps);
    }
    __syncthreads();
    const float inv = red[0];
    for (int k = threadIdx.x; k < K; k += blockDim.x)
        out[blockIdx.x * ldo + k] = __float2bfloat16_rn(__bfloat162float(xr[k]) * inv * __bfloat162float(g[k]));
}

__global__ void silu_mul_kernel(const __nv_bfloat16* __restrict__ g, int64_t ldg, const __nv_bfloat16* __restrict__ u,
                                int64_t ldu, __nv_bfloat16* __restrict__ out, int64_t ldo, int M, int N) {
    const int64_t total = int64_t(M) * N;
    for (int64_t idx = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; idx < total;
         idx += int64_t(gridDim.x) * blockDim.x) {
        const int m = int(idx / N), n = int(idx % N);
        const float gv = __bfloat162float(g[m * ldg + n]);
        out[m * ldo + n] = __float2bfloat16_rn(silu(gv) * __bfloat162float(u[m * ldu + n]));
    }
}

static int grid_for(int64_t work, int threads) {
    const DeviceInfo* di = device_info();
    const int64_t want = (work + threads - 1) / threads;
    const int64_t cap = di ? int64_t(di->sm_count) * 16 : 2048;
    return int(want < 1 ? 1 : (want > cap ? cap : want));
}

static int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "%s launch failed: %s", what, cudaGetErrorString(e));
    return BQ_OK;
}


// One CTA per output row: out[r] = table[clamp(ids[r * ld_ids] + offset, 0, rows - 1)].
__global__ void embed_rows_kernel(const uint8_t* __restrict__ table, int64_t ld_bytes, int64_t table_rows,
                                  const int64_t* __restrict__ ids, int64_t ld_ids, int64_t offset, int width_bytes,
                                  uint8_t* __restrict__ out, int64_t ldo_bytes, int vec) {
    pdl_launch_dependents();
    pdl_wait();  // the ids come from the previous step's sampler
    const int r = blockIdx.x;
    int64_t row = ids[int64_t(r) * ld_ids] + offset;
    row = row < 0 ? 0 : (row >= table_rows ? table_rows - 1 : row);
    const uint8_t* src = table + row * ld_bytes;
    uint8_t* dst = out + int64_t(r) * ldo_bytes;
    if (vec) {
        for (int i = threadIdx.x; i < width_bytes / 16; i += blockDim.x)
            reinterpret_cast<uint4*>(dst)[i] = __ldg(reinterpret_cast<const uint4*>(src) + i);
    } else {
        for (int i = threadIdx.x; i < width_bytes / 2; i += blockDim.x)
            reinterpret_cast<uint16_t*>(dst)[i] = reinterpret_cast<const uint16_t*>(src)[i];
    }
}

}  // namespace bq

using namespace bq;

extern "C" {

int32_t bq_int4_tinygemm_pack(const void* packed_u8, void* out_i32, int32_t N, int32_t K, int32_t inner_k_tiles,
                              void* stream) {
    if (!packed_u8 || !out_i32) return set_error(BQ_ERR_INVALID_ARG, "NULL tensor");
    if (inner_k_tiles != 2 && inner_k_tiles != 4 && inner_k_tiles != 8)
        return set_error(BQ_ERR_SHAPE, "inner_k_tiles must be 2, 4 or 8 (got %d)", inner_k_tiles);
    if (N <= 0 || N % 8 || K <= 0 || K % (16 * inner_k_tiles))
        return set_error(BQ_ERR_SHAPE, "pack needs N %% 8 == 0 and K %% %d == 0 (got N=%d K=%d)", 16 * inner_k_tiles, N, K);
    const int64_t words = int64_t(N) * K / 8;
    tinygemm_pack_kernel<<<grid_for(words, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint8_t*>(packed_u8), static_cast<uint32_t*>(out_i32), N, K, inner_k_tiles);
    return check_launch("tinygemm pack");
}

int32_t bq_int4_tinygemm_unpack(const void* in_i32, void* packed_u8, int32_t N, int32_t K, int32_t inner_k_tiles,
                                void* stream) {
    if (!packed_u8 || !in_i32) return set_error(BQ_ERR_INVALID_ARG, "NULL tensor");
    if (inner_k_tiles != 2 && inner_k_tiles != 4 && inner_k_tiles != 8)
        return set_error(BQ_ERR_SHAPE, "inner_k_tiles must be 2, 4 or 8 (got %d)", inner_k_tiles);
    if (N <= 0 || N % 8 || K <= 0 || K % (16 * inner_k_tiles))
        return set_error(BQ_ERR_SHAPE, "unpack needs N %% 8 == 0 and K %% %d == 0 (got N=%d K=%d)", 16 * inner_k_tiles, N, K);
    const int64_t words = int64_t(N) * K / 8;
    tinygemm_unpack_kernel<<<grid_for(words, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint32_t*>(in_i32), static_cast<uint8_t*>(packed_u8), N, K, inner_k_tiles);
    return check_launch("tinygemm unpack");
}

int32_t bq_dequant(const bq_gemv_desc* desc, float* out, void* stream) {
    if (!desc || !out || !desc->w) return set_error(BQ_ERR_INVALID_ARG, "NULL argument");
    if (desc->N < 1 || desc->K < 1 || desc->K % 128) return set_error(BQ_ERR_SHAPE, "bad N/K (%d, %d)", desc->N, desc->K);
    if (desc->wfmt < BQ_W_BF16 || desc->wfmt > BQ_W_INT8) return set_error(BQ_ERR_FORMAT, "unknown format %d", desc->wfmt);
    if (desc->wfmt != BQ_W_BF16 && !desc->scale) return set_error(BQ_ERR_INVALID_ARG, "scale is NULL");
    if (desc->wfmt == BQ_W_INT4_TINYGEMM && (desc->N % 8 || desc->group < 32 || desc->K % desc->group))
        return set_error(BQ_ERR_SHAPE, "bad int4 geometry");
    bq_gemv_desc d = *desc;
    if (d.wfmt == BQ_W_INT4_PLAIN) d.group = 128;
    const int64_t total = int64_t(d.N) * d.K;
    dequant_kernel<<<grid_for(total, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(d, out);
    return check_launch("dequant");
}

int32_t bq_rmsnorm(const void* x, int64_t ldx, const void* gamma, void* out, int64_t ldo, int32_t M, int32_t K,
                   float eps, void* stream) {
    if (!x || !gamma || !out) return set_error(BQ_ERR_INVALID_ARG, "NULL tensor");
    if (M < 1 || K < 1 || ldx < K || ldo < K) return set_error(BQ_ERR_SHAPE, "bad rmsnorm shape");
    rmsnorm_kernel<<<M, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(x), ldx, static_cast<const __nv_bfloat16*>(gamma),
        static_cast<__nv_bfloat16*>(out), ldo, K, eps);
    return check_launch("rmsnorm");
}

int32_t bq_silu_mul(const void* g, int64_t ldg, const void* u, int64_t ldu, void* out, int64_t ldo, int32_t M, int32_t N,
                    void* stream) {
    if (!g || !u || !out) return set_error(BQ_ERR_INVALID_ARG, "NULL tensor");
    if (M < 1 || N < 1 || ldg < N || ldu < N || ldo < N) return set_error(BQ_ERR_SHAPE, "bad silu_mul shape");
    silu_mul_kernel<<<grid_for(int64_t(M) * N, 256), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<const __nv_bfloat16*>(g), ldg, static_cast<const __nv_bfloat16*>(u), ldu,
        static_cast<__nv_bfloat16*>(out), ldo, M, N);
    return check_launch("silu_mul");
}

int32_t bq_embed_rows(const void* table, int64_t ld_table, int64_t table_rows, const int64_t* ids, int64_t ld_ids,
                      int64_t offset, int32_t n, int32_t width, void* out, int64_t ldo, uint32_t flags, void* stream) {
    if (!table || !ids || !out) return set_error(BQ_ERR_INVALID_ARG, "table, ids and out must be non-NULL");
    if (n < 1 || width < 1 || table_rows < 1 || ld_table < width || ldo < width)
        return set_error(BQ_ERR_SHAPE, "bad embedding lookup shape (n=%d, width=%d)", n, width);
    const int vec = ((reinterpret_cast<uintptr_t>(table) | reinterpret_cast<uintptr_t>(out)) % 16 == 0 &&
                     (ld_table * 2) % 16 == 0 && (ldo * 2) % 16 == 0 && (int64_t(width) * 2) % 16 == 0)
                        ? 1
                        : 0;
    cudaLaunchConfig_t cfg;
    std::memset(&cfg, 0, sizeof(cfg));
    cfg.gridDim = dim3(n);
    cfg.blockDim = dim3(128);
    cfg.stream = static_cast<cudaStream_t>(stream);
    cudaLaunchAttribute attr[1];
    if (flags & BQ_FLAG_PDL) {
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
    }
    const uint8_t* tb = static_cast<const uint8_t*>(table);
    int64_t ldb = ld_table * 2, tr = table_rows, ldi = ld_ids, off = offset, ldob = ldo * 2;
    int wb = width * 2;
    uint8_t* ob = static_cast<uint8_t*>(out);
    void* args[] = {&tb, &ldb, &tr, &ids, &ldi, &off, &wb, &ob, &ldob, const_cast<int*>(&vec)};
    cudaError_t e = cudaLaunchKernelExC(&cfg, reinterpret_cast<const void*>(&embed_rows_kernel), args);
    if (e != cudaSuccess) return set_error(BQ_ERR_CUDA, "embed launch failed: %s", cudaGetErrorString(e));
    return BQ_OK;
}

}  // extern "C"
