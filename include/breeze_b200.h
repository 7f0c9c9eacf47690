/*
 * breeze_b200.h -- C ABI of the B200-native weight-only quantized decode GEMV.
 *
 * One shared library (libbreeze_b200.so, built for sm_100a) replaces the
 * per-token decode linear layers of the reference:
 *
 *   models/fused/kernels.py:334  rms_gemv(x, fw, norm_weight, eps, epilogue, residual, out)
 *   models/fused/kernels.py:41   rms_gemv_kernel      (RMSNorm prologue + streamed GEMV)
 *   models/fused/kernels.py:107  gemv_epilogue_kernel (split-K sum, fp8 scale, SiLU*up / +residual)
 *   models/int4_linear.py:99     Int4Linear.forward   (torch._weight_int4pack_mm, tinygemm layout)
 *   models/fp8_linear.py:68      Fp8Linear.forward    (torch._scaled_mm)
 *   models/int8_linear.py:50     Int8Linear.forward   (dequant + F.linear)
 *   models/int4_linear.py:59     torch._convert_weight_to_int4pack (int4 re-tiling)
 *   models/fused/kernels.py:541  rmsnorm_kernel, :560 silu_mul_kernel (glue)
 *
 * Conventions
 *   - Plain C types only: device pointers are void*, sizes are int32/int64,
 *     streams are cudaStream_t passed as void*. No torch types.
 *   - Every entry point returns 0 on success or a negative BQ_ERR_* code and
 *     never aborts; bq_last_error_string() describes the last failure of the
 *     calling host thread.
 *   - Nothing here allocates or frees device memory. Scratch space (split-K
 *     partial sums and arrival counters) is a caller-provided workspace of
 *     bq_gemv_workspace_bytes() bytes that must be ZERO-FILLED ONCE before
 *     its first use; every call leaves the counters at zero again. One
 *     workspace must not be used by two calls that can run concurrently.
 *   - Launches are asynchronous on the given stream, take no host
 *     synchronization and keep a fixed grid for fixed shapes, so they can be
 *     captured into CUDA graphs.
 */
#ifndef BREEZE_B200_H
#define BREEZE_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define BQ_VERSION 1

/* ---- status codes ------------------------------------------------------ */
#define BQ_OK 0
#define BQ_ERR_INVALID_ARG -1  /* null pointer where one is required, bad enum */
#define BQ_ERR_SHAPE -2        /* M/N/K/group not supported or inconsistent    */
#define BQ_ERR_ALIGN -3        /* pointer or stride alignment                  */
#define BQ_ERR_FORMAT -4       /* weight format / dtype combination            */
#define BQ_ERR_WORKSPACE -5    /* workspace missing or too small               */
#define BQ_ERR_CUDA -6         /* a CUDA runtime/driver call failed            */
#define BQ_ERR_DEVICE -7       /* device is not sm_100 (B200 class)            */

/* Device-side error bits, read with bq_device_status(). */
#define BQ_DEVERR_WAIT_TIMEOUT 1u /* a bounded device wait gave up */
#define BQ_DEVERR_POSITION 2u     /* bq_attention_step saw a cache position outside [0, S) */

/* ---- enums --------------------------------------------------------------- */
/* Weight formats. */
#define BQ_W_BF16 0          /* w: bf16 [N, K] row-major (FusedWeight bits=16)             */
#define BQ_W_INT4_TINYGEMM 1 /* w: int32 [N/8, K/128, 32, 4] (Int4Linear.weight_int4,
                                innerKTiles=8), scale: bf16 [K/g, N, 2] (scale, zero),
                                w = (q - 8) * scale + zero, g in {32, 64, 128, 256}          */
#define BQ_W_INT4_PLAIN 2    /* w: uint8 [N, K/2] even-k low nibble (FusedWeight bits=4),
                                scale: bf16 [K/128, N, 2] (scale, min), w = q * scale + min  */
#define BQ_W_FP8_E4M3 3      /* w: e4m3 [N, K] row-major, scale: fp32 [N], w = q * scale    */
#define BQ_W_INT8 4          /* w: int8 [N, K] row-major, scale: fp32 [N], w = q * scale    */

/* Epilogues (models/fused/kernels.py:116-137). */
#define BQ_EPI_NONE 0         /* out = acc                                             */
#define BQ_EPI_SILU_MUL 1     /* out[:, n] = silu(acc[:, n]) * acc[:, n + N/2], N/2 outputs */
#define BQ_EPI_ADD_RESIDUAL 2 /* out = acc + residual                                  */

/* Activation / output dtypes. */
#define BQ_DT_BF16 0
#define BQ_DT_F16 1
#define BQ_DT_F32 2

/* Flags. */
#define BQ_FLAG_PDL 1u              /* launch with programmatic dependent launch: weight
                                       streaming starts before the previous kernel ends  */
#define BQ_FLAG_SCALE_ROUND_BF16 2u /* int8: round the per-row scale to bf16 first, as
                                       Int8Linear does for bf16 activations              */
#define BQ_FLAG_NO_TC 4u            /* keep 17..128-row calls on the mma.sync kernel (row
                                       blocks of 16) instead of the tcgen05 kernel        */
#define BQ_FLAG_RING_KERNEL 8u      /* keep one- and two-row calls on the ring-streaming
                                       kernel instead of the resident-slice kernel (for
                                       comparisons; results agree within rounding)       */

typedef struct bq_gemv_desc {
    int32_t M;         /* activation rows (decode batch), >= 1 */
    int32_t N;         /* weight rows = output features (for SILU_MUL: gate+up rows) */
    int32_t K;         /* input features, multiple of 128 */
    int32_t wfmt;      /* BQ_W_* */
    int32_t group;     /* int4 group size (tinygemm: 32/64/128/256; plain: 128) */
    int32_t epilogue;  /* BQ_EPI_* */
    int32_t x_dtype;   /* BQ_DT_* */
    int32_t out_dtype; /* BQ_DT_* */
    int32_t res_dtype; /* BQ_DT_* (residual) */
    uint32_t flags;    /* BQ_FLAG_* */
    float eps;         /* RMSNorm epsilon (used when gamma != NULL) */
    int32_t reserved;
    const void* x;        /* [M, ldx] activations (the residual stream when gamma != NULL) */
    int64_t ldx;          /* row stride of x, elements */
    const void* gamma;    /* bf16 [K] RMSNorm weight, or NULL for no norm */
    const void* w;        /* packed weights, 16-byte aligned */
    const void* scale;    /* see BQ_W_* */
    const void* bias;     /* [N] in out_dtype (the output's element type), or NULL */
    const void* residual; /* [M, ldr] for BQ_EPI_ADD_RESIDUAL, else NULL */
    int64_t ldr;
    void* out;            /* [M, ldo] */
    int64_t ldo;
} bq_gemv_desc;

/* ---- library ----------------------------------------------------------- */
int32_t bq_version(void);
const char* bq_last_error_string(void);

/* Device-side error bits accumulated by the kernels on `device` since the
 * last clear (blocking read; not for use inside stream capture). */
int32_t bq_device_status(int32_t device, uint32_t* bits);
int32_t bq_device_status_clear(int32_t device);

/* ---- GEMV (replaces rms_gemv / Int4Linear / Fp8Linear / Int8Linear) ------ */
/* Workspace bytes needed by bq_gemv for `desc` on the current device. */
int32_t bq_gemv_workspace_bytes(const bq_gemv_desc* desc, size_t* bytes);

/* out = epilogue( rmsnorm(x) @ dequant(w)^T ), fp32 accumulation.
 * Replaces models/fused/kernels.py:334-351 (rms_gemv + both kernels),
 * models/int4_linear.py:99-109, models/fp8_linear.py:68-83 (weight-only),
 * models/int8_linear.py:50-53.
 * Two kernels: up to 16 rows per pass on mma.sync tiles with in-register
 * dequantization (more rows: passes of 16, each streaming the weights again);
 * 17..128 bf16 rows with N % 128 == 0 on tcgen05 tiles (dequantized weights
 * in tensor memory, the rows in shared memory, weights read once; with an
 * RMSNorm the normalized rows go through the workspace first) unless
 * BQ_FLAG_NO_TC is set. */
int32_t bq_gemv(const bq_gemv_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* bq_gemv with host-side input and output: x_host (M rows of K values, dense,
 * x_dtype) is copied into desc->x, the GEMV runs, and the output (M rows of
 * N, or N / 2 with the SiLU epilogue, dense, out_dtype) is copied from
 * desc->out into out_host, all enqueued on `stream` (pinned host memory makes
 * the copies asynchronous); the call does not wait. Replaces rms_gemv
 * (models/fused/kernels.py:334-351) on tensors that the caller moves to the
 * device and back around it. */
int32_t bq_gemv_host_io(const bq_gemv_desc* desc, const void* x_host, void* out_host, void* workspace,
                        size_t workspace_bytes, void* stream);

/* bq_gemv for callers that cannot allocate device memory (fixed VRAM
 * budgets, hosts that own every allocation, real-time threads that must not
 * call cudaMalloc/cudaFree). No counterpart in the reference. The same kernel
 * and launch plan as bq_gemv, with one 4 MiB scratch array built into the
 * library (held by every GPU that loads it until exit) in place of the
 * caller's workspace; shapes whose bq_gemv_workspace_bytes exceed it return
 * BQ_ERR_WORKSPACE without launching. The first call on a device (and the
 * first after a cudaDeviceReset) clears the array's counters with a blocking
 * memset: make it before any stream capture. All calls on a device share the
 * array: calls whose kernels can overlap on the GPU race and must be
 * serialized on one stream. For more than 16 rows, when the tensor-core
 * kernel's split-K pieces would not fit the array, the call runs the 16-row
 * block kernel instead, whose summation order differs from the tensor-core
 * kernel that bq_gemv then uses (results agree within rounding, not bit for
 * bit). After a device wait timeout, bq_device_status_clear on that device
 * makes the next call clear the counters again (blocking, outside capture).
 * The array's address is looked up on every call, so after a
 * cudaDeviceReset the next call finds the reloaded array and clears it. */
int32_t bq_gemv_noalloc(const bq_gemv_desc* desc, void* stream);

/* ---- decode chain: a list of GEMVs in one launch ------------------------ */
/* Runs descs[0..n) in order as ONE persistent cooperative launch, one CTA per
 * SM: a producer warp per CTA streams the weights of the CTA's share of every
 * GEMV through a shared-memory ring with bulk copies, running ahead across
 * GEMV boundaries, while eight consumer warps compute each GEMV as soon as
 * the previous one is complete (per-GEMV completion counters in the
 * workspace; no grid barrier). Replaces the per-projection rms_gemv /
 * Int4Linear launches of one decode step (models/fused/layer.py:87-98 over
 * every layer, as captured by cudagraph/backbone_graph.py:254-285); GEMV i
 * may read the output of any earlier GEMV. Every GEMV of a chain has the same
 * M (<= 16); formats, groups and epilogues may differ. Each needs bf16 x with
 * 16-byte aligned rows, N (N / 2 with SiLU*up) a multiple of 16, a bf16
 * residual with 16-byte aligned rows, 16-byte aligned gamma and row scales
 * (BQ_ERR_SHAPE / BQ_ERR_ALIGN otherwise).
 * The workspace (size from bq_gemv_chain_workspace_bytes, 256-byte aligned)
 * holds the op table, the completion counters and a tile-major copy of every
 * int4 GEMV's scale/zero pairs: bq_gemv_chain_prepare writes it
 * (synchronously, outside stream capture), after which bq_gemv_chain_launch
 * is capture-safe and may be replayed. Re-prepare when any pointer in the
 * descriptors, or the contents of an int4 scale tensor, change, and after a
 * launch that set a device error bit (its counters are then inconsistent).
 * No counterpart in the reference. */
typedef struct bq_chain_options {
    uint64_t wait_cycles;        /* bound of every device-side wait in SM clock cycles; 0: ~2 s */
    const uint32_t* start_flag;  /* NULL, or a word the device can read (device memory or mapped host
                                  * memory) written by the host or by work finished before the launch
                                  * -- never by a kernel running at the same time: the first GEMV also
                                  * waits until *start_flag >= start_target */
    uint32_t start_target;
} bq_chain_options;

int32_t bq_gemv_chain_workspace_bytes(const bq_gemv_desc* descs, int32_t n, size_t* bytes);
int32_t bq_gemv_chain_prepare(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes);
/* bq_gemv_chain_prepare with options (NULL: the defaults). A wait that runs
 * out sets BQ_DEVERR_WAIT_TIMEOUT in bq_device_status; the kernel then stops
 * at its next wait, lets its copies in flight land, and returns. */
int32_t bq_gemv_chain_prepare_ex(const bq_gemv_desc* descs, int32_t n, const bq_chain_options* opts, void* workspace,
                                 size_t workspace_bytes);
int32_t bq_gemv_chain_launch(const bq_gemv_desc* descs, int32_t n, void* workspace, size_t workspace_bytes,
                             void* stream);

/* ---- decode attention step --------------------------------------------- */
/* One decode step of attention for a static KV cache: per-head RMSNorm of q
 * and k (when q_norm / k_norm are given), RoPE (rotate_half), the new k and v
 * written into the caches at *pos, then softmax((q * D^-0.5) k^T + mask) v
 * over cache positions [0, *pos] with grouped-query heads (q head h reads kv
 * head h / (HQ / HKV)). Replaces attention_step and its three Triton
 * kernels (models/fused/kernels.py:376-536), called from
 * FusedDecoderLayer.forward (models/fused/layer.py:89-90). */
typedef struct bq_attn_desc {
    int32_t B, HQ, HKV, D, S;   /* batch rows, q heads, kv heads, head dim (64 or 128), cache length */
    int32_t mask_dtype;         /* BQ_DT_BF16 or BQ_DT_F32; additive (B, S) mask, may be NULL */
    float eps;                  /* RMSNorm epsilon */
    uint32_t flags;             /* BQ_FLAG_PDL */
    const void* qkv;            /* (B, (HQ + 2 HKV) D) bf16: [q heads | k heads | v heads] */
    int64_t ldqkv;
    const void* cos;            /* (B or 1, D) bf16 */
    const void* sin;
    int64_t ldcs;               /* row stride of cos / sin; 0 broadcasts one row */
    const int64_t* pos;         /* device pointer to the cache position */
    void* k_cache;              /* (B, HKV, S, D) bf16, written at pos */
    void* v_cache;
    const void* mask;
    int64_t ldm;
    const void* q_norm;         /* (D) bf16 or NULL */
    const void* k_norm;
    void* out;                  /* (B, HQ D) bf16 */
    int64_t ldo;
} bq_attn_desc;

/* The workspace (256-byte aligned) starts with arrival counters that the
 * kernel leaves at zero; do not share it with bq_gemv's workspace, whose own
 * counters must stay zero between calls. */
int32_t bq_attention_workspace_bytes(const bq_attn_desc* desc, size_t* bytes);
int32_t bq_attention_step(const bq_attn_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* ---- attention step fused with the output projection ------------------- */
/* out = residual + attention_step(attn) @ wo^T, for short caches (S <= 256,
 * B <= 4; the additive mask as in bq_attention_step): replaces the reference FusedDecoderLayer's
 * attention_step followed by rms_gemv(attn, wo, None, epilogue=2,
 * residual=x) (models/fused/layer.py:89-91) with bf16 wo, as the depth
 * decoder runs them (attn_bits=16). The attention output is rounded to bf16
 * as the unfused step stores it and never leaves the chip; the caches are
 * written as by bq_attention_step. attn.out / attn.ldo are ignored. */
typedef struct bq_attn_o_desc {
    bq_attn_desc attn;
    int32_t N;                 /* O outputs (multiple of 16) */
    int32_t reserved;
    const void* wo;            /* bf16 [N, ldw], K = HQ D columns; 16-byte aligned rows */
    int64_t ldw;
    const void* residual;      /* bf16 [B, ldr] */
    int64_t ldr;
    void* out;                 /* bf16 [B, ldo] */
    int64_t ldo;
} bq_attn_o_desc;

/* The workspace (256-byte aligned) starts with arrival counters that the
 * kernel leaves at zero; it may be shared with bq_attention_step's. */
int32_t bq_attention_o_workspace_bytes(const bq_attn_o_desc* desc, size_t* bytes);
int32_t bq_attention_o_step(const bq_attn_o_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* ---- fp32 output heads -------------------------------------------------- */
/* out[M, N] (fp32) = y @ W, W fp32, where y is x or, when gamma is given, the
 * reference's BreezeRMSNorm of x (models/breeze.py:115-120: xh = bf16(x *
 * rsqrt(mean(x^2) + eps)), y = bf16(gamma * xh)) read as fp32.
 * Replaces the fp32 heads of the decode graphs: BreezeCodebooksHead.forward
 * (models/breeze.py:598-613; W = weight[codebook], layout K-major) after the
 * depth model's final norm (models/cudagraph/depth_decoder_graph.py:161,
 * 617-623, 641-648), and the backbone lm_head.float() (nn.Linear weight,
 * layout N-major; models/cudagraph/backbone_graph.py:70, 272-273). */
#define BQ_HEAD_NK 0 /* W[n * ldw + k]: nn.Linear weight [N, K]               */
#define BQ_HEAD_KN 1 /* W[k * ldw + n]: one codebook slice [K, N] (hidden, vocab) */

typedef struct bq_head_desc {
    int32_t M, N, K;     /* rows (M <= 16), outputs, inputs */
    int32_t layout;      /* BQ_HEAD_NK or BQ_HEAD_KN */
    int32_t x_dtype;     /* BQ_DT_* */
    uint32_t flags;      /* BQ_FLAG_PDL */
    float eps;           /* RMSNorm epsilon (gamma != NULL) */
    int32_t reserved;
    const void* x;       /* [M, ldx] */
    int64_t ldx;
    const void* gamma;   /* bf16 [K] or NULL */
    const float* w;      /* fp32, see layout */
    int64_t ldw;
    float* out;          /* fp32 [M, ldo] */
    int64_t ldo;
} bq_head_desc;

/* The workspace (K-major layout only; 256-byte aligned) starts with arrival
 * counters that the kernel leaves at zero: zero-fill it once, and give it to
 * no other kernel. */
int32_t bq_head_workspace_bytes(const bq_head_desc* desc, size_t* bytes);
int32_t bq_head_gemv(const bq_head_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* ---- CFG mix and token sampling ----------------------------------------- */
/* Per sample row r: cfg = uncond + g * (cond - uncond) (paired rows; else cond),
 * logits [mask_lo, mask_hi) = -inf (mask_invalid_codec_token_logits), the
 * HF repetition penalty over the row's token history, the suppress mask;
 * greedy = argmax(cfg); then temperature, top-k, top-p (HF order, on raw
 * logits), softmax and one draw by inverse CDF over the kept tokens in
 * descending-probability order with u in [0, 1); token = do_sample ? draw :
 * greedy, clamped to [0, clamp_hi]. u comes from `uniform` or from
 * Philox4x32-10 (key = rng[0], counter = {rng[1], r}); the launch advances
 * rng[1] by one, so a replayed graph draws fresh numbers.
 * Replaces DepthDecoderGraph._cfg_sample (models/cudagraph/depth_decoder_graph.py:
 * 487-558) and sample_logits (models/cudagraph/sampling.py:36-87) with the CFG
 * mix of BackboneGraph._decode_step (models/cudagraph/backbone_graph.py:275-285). */
#define BQ_SAMPLE_TOPK_VALUE 2u /* top-k keeps every logit >= the k-th largest (sample_logits);
                                   default: the first k ranks (the depth graph's topk mask)   */
#define BQ_SAMPLE_APPEND_HISTORY 4u /* before sampling, append the row's current token
                                       (tokens[r * ldt]) to its history, as the backbone
                                       loop does with the previous step's token
                                       (models/fast_streaming.py:929-939)          */
#define BQ_SAMPLE_MAX_V 8192

typedef struct bq_sample_desc {
    int32_t rows;              /* samples; with cfg the logits hold 2 * rows rows: cond, then uncond */
    int32_t V;                 /* logits per row, <= BQ_SAMPLE_MAX_V */
    int32_t cfg;               /* 0 or 1 */
    int32_t max_k;             /* top_k <= 0 means max_k; top_k is clamped to [1, max_k] */
    int32_t mask_lo, mask_hi;  /* logits [mask_lo, mask_hi) become -inf (empty when equal) */
    int32_t clamp_hi;          /* tokens are clamped to [0, clamp_hi] */
    uint32_t flags;            /* BQ_FLAG_PDL | BQ_SAMPLE_TOPK_VALUE */
    float rep_penalty;         /* HF repetition penalty (1 = none) */
    int32_t history_cap;       /* tokens per history row */
    const float* logits;       /* fp32 [rows or 2 rows, ldl] */
    int64_t ldl;
    const float* guidance;     /* fp32 [rows] (cfg only) */
    const float* temperature;  /* fp32 [rows] */
    const int64_t* top_k;      /* int64 [rows] */
    const float* top_p;        /* fp32 [rows] */
    const int64_t* do_sample;  /* int64 [rows], 0 = greedy */
    int64_t* history;          /* int64 [rows, history_cap] or NULL */
    int32_t* history_len;      /* int32 [rows] valid entries per history row */
    const uint8_t* suppress;   /* bool [V] or NULL */
    const float* uniform;      /* fp32 [rows] or NULL (Philox) */
    uint64_t* rng;             /* {seed, call counter}, required when uniform is NULL */
    float* cfg_out;            /* fp32 [rows, ldc] mixed and masked logits, or NULL */
    int64_t ldc;
    int64_t* tokens;           /* tokens[r * ldt]; with cfg also tokens[(r + rows) * ldt] */
    int64_t ldt;
    int64_t* tokens2;          /* optional second destination, same rule */
    int64_t ldt2;
    int64_t eos_id;            /* token that sets *eos_flag (the backbone EOS class), or -1 */
    int32_t* eos_flag;         /* set to 1 when a row draws eos_id; never cleared here; or NULL */
} bq_sample_desc;

/* 256 bytes (an arrival counter the kernel leaves at zero); zero-fill once. */
int32_t bq_sample_workspace_bytes(const bq_sample_desc* desc, size_t* bytes);
int32_t bq_sample(const bq_sample_desc* desc, void* workspace, size_t workspace_bytes, void* stream);

/* ---- layouts and dequantization ---------------------------------------- */
/* (N, K/2) uint8 odd-k-low -> tinygemm int32 [N/8, K/(16*ikt), 32, ikt/2].
 * Replaces torch._convert_weight_to_int4pack (models/int4_linear.py:59). */
int32_t bq_int4_tinygemm_pack(const void* packed_u8, void* out_i32, int32_t N, int32_t K,
                              int32_t inner_k_tiles, void* stream);
/* Inverse of bq_int4_tinygemm_pack (tinygemm int32 -> (N, K/2) uint8). */
int32_t bq_int4_tinygemm_unpack(const void* in_i32, void* packed_u8, int32_t N, int32_t K,
                                int32_t inner_k_tiles, void* stream);

/* Dequantized weights W[N, K] as fp32, bit-exact with the reference's
 * dequantization (int4: fmaf((q-8), s, z) / fmaf(q, s, min); fp8: q * s;
 * int8: bf16(bf16(q) * bf16(s)); bf16: the value). Uses desc->{N, K, wfmt,
 * group, w, scale}. For parity checks and debugging. */
int32_t bq_dequant(const bq_gemv_desc* desc, float* out, void* stream);

/* ---- embedding lookup ---------------------------------------------------- */
/* out[r, :] = table[clamp(ids[r * ld_ids] + offset, 0, table_rows - 1), :] for
 * r < n; bf16 rows of `width` elements. The depth loop's token embedding
 * (embed_tokens(tok + codebook offset), clamped:
 * models/cudagraph/depth_decoder_graph.py:563-567, 602-609). ids are read
 * after the dependent-launch wait (they come from the previous sampler). */
int32_t bq_embed_rows(const void* table, int64_t ld_table, int64_t table_rows, const int64_t* ids, int64_t ld_ids,
                      int64_t offset, int32_t n, int32_t width, void* out, int64_t ldo, uint32_t flags, void* stream);

/* ---- glue kernels (models/fused/kernels.py:541-575) ---------------------- */
/* out[M, K] = x * rsqrt(mean(x^2) + eps) * gamma (fp32 math), bf16 in/out. */
int32_t bq_rmsnorm(const void* x, int64_t ldx, const void* gamma, void* out, int64_t ldo,
                   int32_t M, int32_t K, float eps, void* stream);
/* out[M, N] = silu(g) * u, bf16 in/out. */
int32_t bq_silu_mul(const void* g, int64_t ldg, const void* u, int64_t ldu, void* out, int64_t ldo,
                    int32_t M, int32_t N, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* BREEZE_B200_H */
