/*
 * ltx_b200.h — C ABI of the B200 (sm_100a) implementation of ltx-rust's
 * denoise-step hot path: FP8 dequant + IC-LoRA merge, the DiT forward, and
 * the Euler/CFG update.
 *
 * Conventions (all entry points):
 *   - Every call returns an `int` status (ltx_status).  Nothing aborts and no
 *     C++ exception crosses this boundary; `ltx_last_error(ctx)` gives the
 *     message of the last failure on that context.  The codes mirror the
 *     reference's error enums (crates/ltx-weights/src/error.rs:7-101,
 *     crates/ltx-dit/src/error.rs, crates/ltx-sampler/src/error.rs).
 *   - Pointers named `*_dev` are CUDA device pointers on the context's device;
 *     the caller owns them.  Handles (ltx_ctx, ltx_store, ltx_model) are owned
 *     by the library and freed with their `*_destroy` call.
 *   - Work is enqueued on the context's stream.  Calls that return host data
 *     synchronise that stream first.
 *   - One ltx_ctx per host thread/stream.  Distinct contexts may be used from
 *     different threads concurrently.  A loaded model is read-only and may be
 *     shared by contexts on the same device.
 */
#ifndef LTX_B200_H
#define LTX_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum {
    LTX_OK = 0,
    LTX_ERR_INVALID_ARG = 1,      /* null pointer, bad enum, bad size                       */
    LTX_ERR_SHAPE = 2,            /* WeightError::LoraShapeMismatch / InvalidTensorData,
                                     DitError shape checks (load.rs:112-135)                */
    LTX_ERR_DTYPE = 3,            /* WeightError::UnsupportedDtype                          */
    LTX_ERR_MISSING_KEY = 4,      /* WeightError::MissingKey                                */
    LTX_ERR_DUPLICATE_KEY = 5,    /* WeightError::DuplicateKey                              */
    LTX_ERR_LORA_RANK = 6,        /* WeightError::LoraRankMismatch                          */
    LTX_ERR_NO_LORA_MATCHES = 7,  /* WeightError::NoLoraMatches                             */
    LTX_ERR_IO = 8,               /* WeightError::Io                                        */
    LTX_ERR_FORMAT = 9,           /* WeightError::Safetensors / ConfigParse                 */
    LTX_ERR_CONFIG = 10,          /* DitError::Config (config.rs:188-231)                   */
    LTX_ERR_SIGMA = 11,           /* SamplerError::InvalidSigma (loop_.rs:126-137)          */
    LTX_ERR_SCHEDULE = 12,        /* SamplerError::EmptySchedule                            */
    LTX_ERR_CUDA = 13,            /* a CUDA runtime or driver call failed                   */
    LTX_ERR_NCCL = 14,            /* a collective failed                                    */
    LTX_ERR_TIMEOUT = 15,         /* a device-side wait gave up (kernel returned early)     */
    LTX_ERR_OOM = 16,             /* device or host allocation failed                       */
    LTX_ERR_UNSUPPORTED = 17,     /* a configuration this build does not implement          */
    LTX_ERR_MISSING_CONFIG = 18,  /* WeightError::MissingConfig                             */
    LTX_ERR_NEGATIVE_CONTEXT = 19 /* SamplerError::MissingNegativeContext                   */
} ltx_status;

/* Element types, named after the safetensors dtype strings. */
typedef enum {
    LTX_F32 = 0,
    LTX_F16 = 1,
    LTX_BF16 = 2,
    LTX_F8_E4M3 = 3,   /* float8_e4m3fn: no infinities, 0x7F/0xFF are NaN */
    LTX_F8_E5M2 = 4
} ltx_dtype;

typedef struct ltx_ctx ltx_ctx;

/* ── context ──────────────────────────────────────────────────────────────── */

/* Creates a context on CUDA device `device` that enqueues on `stream` (a
 * cudaStream_t owned by the caller; NULL = the CUDA default stream).  No
 * reference counterpart: the reference picks its device through Burn's
 * `B::Device`. */
int ltx_ctx_create(int device, void *stream, ltx_ctx **out);
void ltx_ctx_destroy(ltx_ctx *ctx);
/* Message of the last failed call on this context ("" if none). */
const char *ltx_last_error(const ltx_ctx *ctx);
/* The cudaStream_t the context enqueues on. */
void *ltx_ctx_stream(const ltx_ctx *ctx);
/* Blocks until the context's stream is idle, then reports any device-side
 * timeout flag a kernel raised (LTX_ERR_TIMEOUT) and clears it. */
int ltx_ctx_synchronize(ltx_ctx *ctx);

/* ── ltx-weights: dequant + LoRA merge ────────────────────────────────────── */

/* One factored LoRA update `coeff * (B @ A)` (LowRankDelta,
 * crates/ltx-weights/src/store.rs:756-763).  A and B stay in their stored
 * dtype (F32/F16/BF16/F8_*); the kernel decodes them exactly to f32, as
 * decode_lora_bytes does (crates/ltx-weights/src/lora.rs:176-209). */
typedef struct {
    const void *a_dev;   /* [rank, in_features] */
    const void *b_dev;   /* [out_features, rank] */
    int32_t rank;
    int32_t a_dtype;     /* ltx_dtype */
    int32_t b_dtype;     /* ltx_dtype */
    float coeff;         /* strength * alpha / rank, see ltx_lora_coeff */
} ltx_lora_delta;

/* Maximum number of stacked LoRA deltas one ltx_dequant_merge call applies. */
#define LTX_MAX_DELTAS 8

/* The per-delta coefficient exactly as merge_lora computes it:
 * fma(strength, alpha / rank, 0) (crates/ltx-weights/src/store.rs:606-615).
 * Pass alpha = rank when the LoRA file has no `.alpha` tensor. */
float ltx_lora_coeff(float strength, float alpha, int32_t rank);

/* Replaces WeightStore::read's numeric body for one [out, in] tensor
 * (crates/ltx-weights/src/store.rs:479-521 + LowRankDelta::add_to :767-793):
 *   v = decode(w)                                 (fp8.rs:90-158 for FP8)
 *   if FP8 and has_scale: v = fma(scale, v, +0)   (store.rs:505-507)
 *   for each delta in order, for each row o, for r = 0..rank-1:
 *       c = coeff * B[o][r];  v[o][i] = fma(c, A[r][i], v[o][i])
 *   dst = v as F32, or as BF16 rounded to nearest-even.
 * Bit-exact with the reference for every input, NaN compared as NaN.
 * `w_dev` has dtype `w_dtype`; `dst_dev` is F32 or BF16 (`dst_dtype`).
 * Runs on the context stream; returns without synchronising. */
int ltx_dequant_merge(ltx_ctx *ctx, const void *w_dev, int32_t w_dtype, int32_t has_scale,
                      float scale, int64_t out_features, int64_t in_features,
                      const ltx_lora_delta *deltas, int32_t n_deltas, void *dst_dev,
                      int32_t dst_dtype);

/* ── ltx-dit: building blocks ─────────────────────────────────────────────── */

/* Epilogues of ltx_gemm_bf16. */
typedef enum {
    LTX_EPI_BF16 = 0,       /* out(bf16) = acc + bias                                  */
    LTX_EPI_GELU_BF16 = 1,  /* out(bf16) = gelu_tanh(acc + bias)  (feed_forward.rs:38-42) */
    LTX_EPI_F32 = 2,        /* out(f32)  = acc + bias                                  */
    LTX_EPI_RESID = 3       /* out(f32) += (acc + bias) * gate[gate_idx[row]][col]
                               (block.rs:138, :152; gate NULL = no gate, block.rs:148) */
} ltx_epilogue;

/* out = epilogue(A[m,k] . W[n,k]^T) on the tensor cores (tcgen05, bf16 in,
 * f32 accumulate).  Replaces Burn `Linear::forward` (y = x W^T + b) for the
 * DiT's projections (attention.rs:150-152, :194; feed_forward.rs:38-42;
 * model.rs:187, :254).  A and W are bf16 row-major with leading dimensions
 * lda/ldw in elements (multiples of 8; 16-byte aligned base pointers).
 * `bias_dev` is f32 [n] or NULL.  For LTX_EPI_RESID, `gate_dev` is f32
 * [U, ld_gate] and `gate_idx_dev` int32 [m] selects the gate row per output
 * row (NULL = row 0).  Enqueued on the context stream. */
int ltx_gemm_bf16(ltx_ctx *ctx, const void *a_dev, int64_t lda, const void *w_dev, int64_t ldw,
                  int32_t m, int32_t n, int32_t k, int32_t epilogue, const float *bias_dev,
                  void *out_dev, int64_t ldo, const float *gate_dev, const int32_t *gate_idx_dev,
                  int64_t ld_gate);

/* out = softmax(q k^T * scale) v per batch and head, without materialising
 * the scores (flash attention on tcgen05; scores and P.V accumulate in TMEM).
 * Replaces sdp_attention / chunked_sdp_attention (attention.rs:228-285,
 * mask = None as in alpha_gen).  q/k/v/out are bf16, token-major: row
 * b*T + t, head h in columns [h*head_dim, (h+1)*head_dim), leading
 * dimensions in elements (multiples of 8, 16-byte aligned bases).  q has
 * tq rows per batch, k/v tk rows.  head_dim must be 128
 * (LTX_ERR_UNSUPPORTED otherwise). */
int ltx_attention_fwd(ltx_ctx *ctx, const void *q_dev, int64_t ldq, const void *k_dev, int64_t ldk,
                      const void *v_dev, int64_t ldv, int32_t batch, int32_t heads, int32_t tq,
                      int32_t tk, int32_t head_dim, float scale, void *out_dev, int64_t ldo);

#ifdef __cplusplus
}
#endif

#endif /* LTX_B200_H */
