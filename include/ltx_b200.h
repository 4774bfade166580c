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
 *     shared by contexts on the same device, except one loaded with
 *     "offload_blocks" > 0: its device block slots are shared state, so it
 *     runs on one context at a time.
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
    LTX_ERR_NEGATIVE_CONTEXT = 19, /* SamplerError::MissingNegativeContext                  */
    LTX_ERR_CHUNK_PLAN = 20,      /* ChunkError (crates/ltx-chunk/src/error.rs)             */
    LTX_ERR_TARGET_TOKENS = 21,   /* SamplerError::TargetTokensTooLarge (loop_.rs:162-185)  */
    LTX_ERR_STRENGTH = 22         /* SamplerError::InvalidStrength (conditioning.rs:150-152) */
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
/* Stores and models made on a context are destroyed before it. */
void ltx_ctx_destroy(ltx_ctx *ctx);
/* Message of the last failed call on this context ("" if none). */
const char *ltx_last_error(const ltx_ctx *ctx);
/* Message of the last failed host-only call (one taking no context, e.g.
 * ltx_chunk_plan) on the calling thread ("" if none). */
const char *ltx_host_last_error(void);
/* The cudaStream_t the context enqueues on. */
void *ltx_ctx_stream(const ltx_ctx *ctx);
/* Blocks until the context's stream is idle, then reports any device-side
 * timeout flag a kernel raised (LTX_ERR_TIMEOUT) and clears it. */
int ltx_ctx_synchronize(ltx_ctx *ctx);

/* ── tensor parallelism ───────────────────────────────────────────────────── */

/* One model split over several GPUs (one process or thread per GPU): the
 * heads of every attention and the FFN's hidden units are divided among the
 * ranks, and each block's three output projections end in a sum-allreduce.
 * No reference counterpart (the reference runs one device).  Flow:
 *   rank 0: ltx_comm_unique_id(id); send id to the other ranks (any channel)
 *   every rank: ltx_ctx_init_comm(ctx, id, nranks, rank)     (collective)
 *   every rank: ltx_model_load / ltx_model_init_random on that context: the
 *               model keeps only this rank's shard
 *   every rank: the same ltx_model_forward / ltx_denoise_step / ltx_denoise_loop
 *               calls with the same inputs; outputs are replicated.
 * The communicator is NCCL, loaded at run time (the copy the process already
 * has, else libnccl.so.2); LTX_ERR_NCCL when it is unavailable or fails. */
#define LTX_COMM_ID_BYTES 128
/* Host-only: a fresh communicator id into id_out (len >= LTX_COMM_ID_BYTES). */
int ltx_comm_unique_id(uint8_t *id_out, size_t len);
/* Collective over the nranks contexts: binds this context to rank `rank`. */
int ltx_ctx_init_comm(ltx_ctx *ctx, const uint8_t *id, size_t len, int32_t nranks, int32_t rank);
/* CFG-parallel pair: the conditional and unconditional passes of the CFG
 * batch (guidance.rs:126, :147) run on two contexts (two GPUs, or two
 * tensor-parallel groups of equal size) instead of as one batch-2 forward.
 * Collective over the 2 ranks of the pair, with an id made by
 * ltx_comm_unique_id: cfg_rank 0 computes the conditional pass, 1 the
 * unconditional one.  ltx_denoise_step / ltx_denoise_loop on such a context
 * run their own pass (batch 1), all-gather the two velocities over the pair
 * once per step, and every rank computes the same CFG/Euler update, so the
 * latents stay identical on all ranks.  Combined with ltx_ctx_init_comm,
 * ranks r and r + n/2 of n GPUs form the pairs and each half is one
 * tensor-parallel group of n/2.  No reference counterpart (the reference runs
 * one device). */
int ltx_ctx_init_cfg_comm(ltx_ctx *ctx, const uint8_t *id, size_t len, int32_t cfg_rank);
/* How the tensor-parallel ranks sum each row-split projection, as set up by
 * the first forward on the context: 0 not yet (or one rank), 1 inside the
 * GEMM over NVLink peer memory (the ranks map each other's memory through
 * CUDA IPC; each rank owns a contiguous range of rows, and the GEMM's
 * epilogue pushes partial products to the rows' owner, which adds them and
 * updates its residual rows and writes them into every rank's residual; from
 * 4 ranks at inner dimension 4096 every norm instead runs on the owner's rows
 * only and the normalised rows are gathered into every rank, which
 * LTX_TP_SEQ_NORMS=1 / =0 in every rank's environment forces on / off), 2 NCCL
 * allreduce (when a rank cannot map its peers, more than 8 ranks, or
 * LTX_TP_EXCHANGE=nccl in every rank's environment).  With 1, a rank's
 * kernels wait on the other ranks' kernels on the device for at most 2 s each
 * (then LTX_ERR_TIMEOUT at the next ltx_ctx_synchronize): every rank must
 * enqueue the same calls within about a second of the others. */
int ltx_ctx_tp_exchange(const ltx_ctx *ctx);
/* LTX_ERR_NCCL if the communicator has recorded an asynchronous error. */
int ltx_ctx_comm_check(ltx_ctx *ctx);
/* Aborts the communicator (after a peer failed); the context falls back to
 * one rank and models built on it can no longer run.  (ltx_ctx_destroy of a
 * context whose ranks share peer memory, ltx_ctx_tp_exchange() == 1, waits
 * for every rank to destroy theirs; after a failure abort first.) */
void ltx_ctx_abort_comm(ltx_ctx *ctx);

/* ── device-side signalling ───────────────────────────────────────────────── */

/* Enqueues on the context's stream a wait until *flag_dev == expect (a
 * 32-bit flag in device memory, possibly a peer GPU's): the stream's later
 * work runs only after another stream or GPU set the flag (ltx_set_flag).
 * The wait is bounded: after timeout_ms (0 or more than 2000 means 2000) it
 * records a code in the context's timeout flag and returns, so a peer that
 * never signals is reported by ltx_ctx_synchronize as LTX_ERR_TIMEOUT and the
 * context stays usable.  No reference counterpart (the reference is one
 * device, ordered by the host). */
int ltx_wait_flag(ltx_ctx *ctx, const int32_t *flag_dev, int32_t expect, uint32_t timeout_ms);
/* Enqueues a release store of `value` to *flag_dev on the context's stream. */
int ltx_set_flag(ltx_ctx *ctx, int32_t *flag_dev, int32_t value);

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

/* Maximum chain scratch, in bytes, that ltx_dequant_merge_noalloc can use. */
#define LTX_NOALLOC_SCRATCH_BYTES (16u << 20)

/* ltx_dequant_merge for callers that cannot allocate device memory — code
 * inside a memory pool or host framework that owns every device allocation,
 * or a process that must not call cudaMalloc after start-up.  No counterpart
 * in the reference (its merge runs on the host).  Same arguments and the same
 * bit-exact result as ltx_dequant_merge, except that it needs no ltx_ctx
 * (creating one allocates): `stream` is a cudaStream_t (NULL = default
 * stream) on the current device, and a failure message is written to
 * `errbuf` (may be NULL).  It calls no cudaMalloc/cudaFree: the merge's chain
 * scratch (4 * total rank * (round_up(in,128) + round_up(out,128)) bytes)
 * lives in one LTX_NOALLOC_SCRATCH_BYTES file-scope device array that every
 * GPU loading the library holds until exit; larger merges return
 * LTX_ERR_UNSUPPORTED before enqueuing anything.  All calls on a device share
 * that array, so calls whose GPU work overlaps (e.g. on two streams) race on
 * it.  The first call on each device looks up the array's device address
 * (cudaGetSymbolAddress) and caches it; make that first call before any
 * stream capture.  The cached address lives as long as the device's primary
 * context: do not call this entry point again after cudaDeviceReset. */
int ltx_dequant_merge_noalloc(void *stream, const void *w_dev, int32_t w_dtype, int32_t has_scale,
                              float scale, int64_t out_features, int64_t in_features,
                              const ltx_lora_delta *deltas, int32_t n_deltas, void *dst_dev,
                              int32_t dst_dtype, char *errbuf, size_t errbuf_len);

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
 * [U, ld_gate] (16-byte aligned rows: ld_gate a multiple of 4) and
 * `gate_idx_dev` int32 [m] selects the gate row per output row (NULL = row
 * 0).  Enqueued on the context stream. */
int ltx_gemm_bf16(ltx_ctx *ctx, const void *a_dev, int64_t lda, const void *w_dev, int64_t ldw,
                  int32_t m, int32_t n, int32_t k, int32_t epilogue, const float *bias_dev,
                  void *out_dev, int64_t ldo, const float *gate_dev, const int32_t *gate_idx_dev,
                  int64_t ld_gate);
/* The same projection with native FP8 operands (tcgen05 kind::f8f6f4, e4m3
 * A and W, f32 accumulate):
 *   acc = A[m,k] . W[n,k]^T  (+ A2[m,k2] . B2[n,k2]^T, bf16, when k2 > 0)
 *   out = epilogue(acc * a_scale[row] * w_scale[col])
 * a_scale_dev: f32 [m] per-row scale of A, or NULL = 1.  w_col_scale_dev: f32
 * [n] per-column weight scale, or NULL = the per-tensor w_scale (e.g. the
 * checkpoint's `{key}_scale`, store.rs:505-507).  The appended bf16 block
 * carries an unmerged low-rank (LoRA) term in the same accumulator: pass
 * A2 = (x . A^T) / a_scale and B2 = coeff * B / w_scale so that the scales
 * cancel (k2 a multiple of 64; 0 = none).  lda/ldw are in bytes = elements
 * (multiples of 16), lda2/ldb2 in elements (multiples of 8).  The north
 * star's FP8 GEMM path (rel-L2 <= 3e-2). */
int ltx_gemm_e4m3(ltx_ctx *ctx, const void *a_dev, int64_t lda, const float *a_scale_dev, const void *w_dev,
                  int64_t ldw, float w_scale, const float *w_col_scale_dev, int32_t m, int32_t n, int32_t k,
                  int32_t epilogue, const float *bias_dev, void *out_dev, int64_t ldo, const float *gate_dev,
                  const int32_t *gate_idx_dev, int64_t ld_gate, const void *a2_dev, int64_t lda2,
                  const void *b2_dev, int64_t ldb2, int32_t k2);

/* Per-row e4m3 quantisation of bf16 rows (the activations of the FP8 GEMM
 * path): scale[row] = amax(row) / 448 (1 for an all-zero row), out = the e4m3
 * bytes of in / scale, round to nearest even, saturating.  cols, ldi and ldo
 * multiples of 8.  No reference counterpart (the reference computes in f32). */
int ltx_quantize_rows_e4m3(ltx_ctx *ctx, const void *in_dev, int64_t ldi, int32_t rows, int32_t cols,
                           void *out_dev, int64_t ldo, float *scale_dev);

/* out = softmax(q k^T * scale) v per batch and head, without materialising
 * the scores (flash attention on tcgen05; scores and P.V accumulate in TMEM).
 * Replaces sdp_attention / chunked_sdp_attention (attention.rs:228-285,
 * mask = None as in alpha_gen).  q/k/out are bf16, v is bf16 or f16
 * (`v_dtype`; with f16 the probabilities P are kept in f16 too), all
 * token-major: row b*T + t, head h in columns [h*head_dim, (h+1)*head_dim),
 * leading dimensions in elements (multiples of 8, 16-byte aligned bases).
 * q has tq rows per batch, k/v tk rows.  head_dim must be 128
 * (LTX_ERR_UNSUPPORTED otherwise). */
int ltx_attention_fwd(ltx_ctx *ctx, const void *q_dev, int64_t ldq, const void *k_dev, int64_t ldk,
                      const void *v_dev, int64_t ldv, int32_t v_dtype, int32_t batch, int32_t heads,
                      int32_t tq, int32_t tk, int32_t head_dim, float scale, void *out_dev, int64_t ldo);

/* ── ltx-weights: the weight store ─────────────────────────────────────────── */

typedef struct ltx_store ltx_store;

/* Key maps applied at open (crates/ltx-weights/src/key_map.rs:90-111). */
#define LTX_KEYMAP_IDENTITY 0     /* KeyMap::identity: names as stored              */
#define LTX_KEYMAP_TRANSFORMER 1  /* KeyMap::transformer: keep and strip
                                     `model.diffusion_model.`                       */

/* WeightStore::open (store.rs:124-208): memory-maps the safetensors files,
 * renames keys, rejects duplicates (LTX_ERR_DUPLICATE_KEY) and hides the
 * `{key}_scale` siblings of FP8 tensors.  __metadata__ is merged, first file
 * wins. */
int ltx_store_open(ltx_ctx *ctx, const char *const *paths, int32_t n_paths, int32_t keymap,
                   ltx_store **out);
void ltx_store_destroy(ltx_store *store);
/* WeightStore::merge_lora (store.rs:542-640): pairs `P.lora_A.weight` /
 * `P.lora_B.weight` with `P.weight`, checks ranks and shapes, alpha defaults
 * to the rank, coeff = ltx_lora_coeff(strength, alpha, rank).  The factors
 * are kept on the device and applied in order by every later read.
 * LTX_ERR_NO_LORA_MATCHES when nothing matched but something was unmatched. */
int ltx_store_merge_lora(ltx_store *store, const char *lora_path, float strength, int32_t *n_matched,
                         int32_t *n_unmatched);
/* WeightStore::contains / keys (store.rs:443-455): 1 if visible, else 0. */
int ltx_store_contains(const ltx_store *store, const char *key);
int32_t ltx_store_num_keys(const ltx_store *store);
const char *ltx_store_key(const ltx_store *store, int32_t index);
/* WeightStore::shape (store.rs:462-467); dtype receives the ltx_dtype or -1. */
int ltx_store_shape(ltx_store *store, const char *key, int64_t *dims, int32_t max_dims, int32_t *ndim,
                    int32_t *dtype);
/* WeightStore::metadata / config (store.rs:425-441): copies the string value
 * (NUL-terminated, truncated to buf_len); *needed = full length + 1. */
int ltx_store_metadata(const ltx_store *store, const char *key, char *buf, size_t buf_len, size_t *needed);
/* WeightStore::read (store.rs:479-521) into device memory: decode, FP8 scale,
 * merged LoRA deltas, as F32 (bit-exact with the reference) or BF16 (its
 * round-to-nearest-even).  Enqueued on the context stream. */
int ltx_store_read(ltx_store *store, const char *key, int32_t dst_dtype, void *dst_dev, size_t dst_bytes);

/* ── ltx-dit: the video transformer ───────────────────────────────────────── */

typedef struct ltx_model ltx_model;

/* VideoTransformer::load (load.rs:61-107) from a store; `config_json` NULL =
 * the store's __metadata__["config"] (bare or under "transformer"), parsed
 * and validated like DiTConfig::from_json (config.rs:176-231).  Linear
 * weights are read through the dequant+merge kernel into bf16; Q|K|V and
 * K|V projections are fused at load.  LTX_ERR_MISSING_KEY / LTX_ERR_SHAPE
 * mirror DitError::Weight.  "offload_blocks": n (0 < n < layers) in the
 * config keeps every block's weights in pinned host memory with n device
 * slots, each block uploaded on a copy stream before use
 * (OffloadMode::Stream, crates/ltx-dit/src/offload.rs:43-56; outputs equal
 * the resident model's). */
int ltx_model_load(ltx_ctx *ctx, ltx_store *store, const char *config_json, ltx_model **out);
/* A random-init model of the given config, built the way an FP8 LTX
 * checkpoint is loaded: every linear weight drawn N(0, 0.02) on the device,
 * quantised to float8_e4m3fn with scale amax/448, and merged with a rank
 * `lora_rank` bf16 LoRA (N(0, 0.01), alpha = rank, `lora_strength`) by the
 * dequant+merge kernel.  No reference counterpart (the reference tests use
 * tiny random-init fixtures). */
int ltx_model_init_random(ltx_ctx *ctx, const char *config_json, uint64_t seed, int32_t lora_rank,
                          float lora_strength, ltx_model **out);
/* Frees the model.  Work that uses it on the callers' streams must have
 * finished (ltx_ctx_synchronize on each context that ran it). */
void ltx_model_destroy(ltx_model *model);
/* Device bytes held by the model's weights. */
int64_t ltx_model_weight_bytes(const ltx_model *model);
/* VideoTransformer::forward (model.rs:169-255) with context_mask and
 * self_attn_mask None (as alpha_gen calls it): latent [B,T,in], timesteps
 * [B,T], positions [B,3,T,2], context [B,S,cross_dim] -> out [B,T,out], all
 * f32 device buffers.  No host round trip: the adaLN path runs once per
 * distinct timestep value, deduplicated on the device into at most 8 tables;
 * a forward with more distinct values is reported as LTX_ERR_UNSUPPORTED by
 * the next ltx_ctx_synchronize (ltx_denoise_step with mask_host has no such
 * limit). */
int ltx_model_forward(ltx_model *model, ltx_ctx *ctx, const float *latent_dev, const float *timesteps_dev,
                      const float *positions_dev, const float *context_dev, int32_t batch, int32_t tokens,
                      int32_t context_tokens, float *out_dev);

/* TransformerBlock::forward (crates/ltx-dit/src/block.rs:118-126, the
 * self-attention / cross-attention / feed-forward body :127-153) for block
 * `block_index` of the model, on the block's own inputs, with context_mask
 * and self_attn_mask None (as alpha_gen calls it):
 *   x_dev        f32 [batch*tokens, D], the residual stream, updated in place
 *   context_dev  f32 [batch*context_tokens, cross_attention_dim]
 *   timestep_dev f32 [batch*tokens, K*D], the per-token modulation the
 *                block's ada_values reads (K = 6, or 9 with cross-attention
 *                adaLN; AdaLayerNormSingle's output, model.rs:196-206)
 *   pe_cos_dev / pe_sin_dev  the RoPE tables as precompute_freqs_cis returns
 *                them (rope.rs:118-167): split, f32 (batch, heads, tokens,
 *                head_dim/2); interleaved, f32 (batch, 1, tokens, D).
 * For a caller that drives the blocks itself (its own loop, offload or
 * inspection).  A model loaded with "offload_blocks" > 0 returns
 * LTX_ERR_UNSUPPORTED here. */
int ltx_block_forward(ltx_model *model, ltx_ctx *ctx, int32_t block_index, float *x_dev, const float *context_dev,
                      const float *timestep_dev, const float *pe_cos_dev, const float *pe_sin_dev, int32_t batch,
                      int32_t tokens, int32_t context_tokens);

/* ── ltx-sampler: one guided Euler step ────────────────────────────────────── */

/* The sampler's update on x0 predictions from any denoiser (a
 * VideoDenoiserModel that is not this DiT, crates/ltx-sampler/src/model.rs:
 * 21-51), on the device:
 *   pred = x0_c + (cfg-1)(x0_c - x0_u), rescaled by
 *          rescale*std(x0_c)/std(pred) + (1-rescale)     (guidance.rs:149-165,
 *          std over all tokens*channels values, tensor3_std :178-195)
 *   x0' = pred*m + clean*(1-m); latent += ((latent - x0')/sigma)(sigma_next - sigma)
 *                                                        (loop_.rs:37-65)
 * cond_x0_dev / uncond_x0_dev / clean_dev / latent_dev f32 [tokens, channels],
 * mask_dev f32 [tokens]; latent_dev is updated in place.  cfg_scale == 1
 * uses the conditional prediction alone (uncond_x0_dev may be NULL).
 * Errors: LTX_ERR_SIGMA (sigma not finite or <= 0, sigma_next not finite or
 * < 0, loop_.rs:126-137), LTX_ERR_NEGATIVE_CONTEXT (cfg_scale != 1 without
 * an unconditional prediction). */
int ltx_cfg_euler_step(ltx_ctx *ctx, const float *cond_x0_dev, const float *uncond_x0_dev, float *latent_dev,
                       const float *clean_dev, const float *mask_dev, int32_t tokens, int32_t channels, float sigma,
                       float sigma_next, float cfg_scale, float rescale_scale);

/* One iteration of euler_denoising_loop (loop_.rs:93-149) around the DiT:
 *   t = mask * sigma per token (guidance.rs:114)
 *   v_c, v_u = DiT(latent, t, positions, ctx_cond / ctx_uncond)  — one batch-2
 *              forward when cfg_scale != 1 (guidance.rs:58-60, :126, :147)
 *   x0 = latent - t * v  (velocity -> x0; the reference has no such adapter,
 *                         this is upstream LTX-2's X0 rule)
 *   pred = x0_c + (cfg-1)(x0_c - x0_u), rescaled by
 *          rescale*std(x0_c)/std(pred) + (1-rescale)  (guidance.rs:149-165)
 *   x0' = x0*m + clean*(1-m); latent += ((latent - x0')/sigma)(sigma_next - sigma)
 *                                                      (loop_.rs:37-65)
 * latent_dev [T, C] is updated in place.  mask_host (optional, T floats, the
 * same values as mask_dev) lets the host size the adaLN tables exactly;
 * without it the timesteps are formed and deduplicated on the device (no host
 * round trip; at most 8 distinct mask values, see ltx_model_forward).
 * LTX_ERR_SIGMA / LTX_ERR_NEGATIVE_CONTEXT as SamplerError::InvalidSigma /
 * MissingNegativeContext. */
int ltx_denoise_step(ltx_model *model, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                     const float *mask_host, const float *mask_dev, const float *positions_dev,
                     const float *ctx_cond_dev, const float *ctx_uncond_dev, int32_t tokens,
                     int32_t context_tokens, float sigma, float sigma_next, float cfg_scale,
                     float rescale_scale);

/* euler_denoising_loop (crates/ltx-sampler/src/loop_.rs:93-149) followed by
 * clear_conditioning (loop_.rs:162-185), all on the device: for each pair
 * (sigmas_host[i], sigmas_host[i+1]) one ltx_denoise_step on latent_dev (in
 * place, [tokens, C]), with no host round trip between steps.  Then the first
 * target_tokens tokens of the final latent are copied to out_dev
 * ([target_tokens, C]; may be NULL to keep only latent_dev).  Errors, checked
 * before anything is enqueued: LTX_ERR_SCHEDULE (fewer than 2 sigmas),
 * LTX_ERR_SIGMA (a step sigma not finite or <= 0, a next sigma not finite or
 * < 0), LTX_ERR_TARGET_TOKENS, LTX_ERR_NEGATIVE_CONTEXT.  The reference
 * checks each sigma pair when it reaches it; since it then returns no state,
 * checking them all first is observably the same. */
int ltx_denoise_loop(ltx_model *model, ltx_ctx *ctx, float *latent_dev, const float *clean_dev,
                     const float *mask_host, const float *mask_dev, const float *positions_dev,
                     const float *ctx_cond_dev, const float *ctx_uncond_dev, int32_t tokens,
                     int32_t context_tokens, const float *sigmas_host, int32_t n_sigmas, float cfg_scale,
                     float rescale_scale, int32_t target_tokens, float *out_dev);
/* GaussianNoiser::apply_with_noise (crates/ltx-sampler/src/noiser.rs:91-106)
 * on the device, in place on latent_dev [tokens, C], bit-exact:
 *   noised = latent * (1 - s) + noise * s
 *   latent = clean * (1 - mask) + noised * mask        (mask per token)
 * The caller supplies the N(0,1) noise (the reference's StdRng stream is
 * host-side and seed-specific; parity fixtures use apply_with_noise too). */
int ltx_apply_noise(ltx_ctx *ctx, float *latent_dev, const float *noise_dev, const float *clean_dev,
                    const float *mask_dev, int32_t tokens, int32_t channels, float noise_scale);

/* ImageKeyframeCondition::apply_to (crates/ltx-sampler/src/conditioning.rs:
 * 127-205) on the device, bit-exact: the tokens of latent frame
 * `latent_frame_index` (tokens_per_frame tokens from latent_frame_index *
 * tokens_per_frame) take the keyframe's tokens in clean_dev [tokens, channels]
 * and 1 - strength in mask_dev [tokens]; every other token keeps its values
 * (each as the reference's clean*keep + image*frame and mask*keep +
 * frame*(1-strength), f32).  image_dev is the one-frame latent
 * [channels, 1, H, W] with H*W = tokens_per_frame, as the reference takes it
 * (patchified inside).  LTX_ERR_STRENGTH for a strength outside [0, 1] (or
 * NaN), LTX_ERR_SHAPE when the frame lies beyond the tokens. */
int ltx_apply_keyframe(ltx_ctx *ctx, float *clean_dev, float *mask_dev, int32_t tokens, int32_t channels,
                       const float *image_dev, int32_t latent_frame_index, int32_t tokens_per_frame, float strength);

/* LTX2Scheduler::execute (crates/ltx-sampler/src/scheduler.rs:67-125): writes
 * steps + 1 sigmas with the reference's f32 operations (bit-exact).  Defaults
 * of SchedulerConfig: max_shift 2.05, base_shift 0.95, stretch 1, terminal 0.1.
 * Host-only; needs no context or GPU. */
int ltx_scheduler_execute(int32_t steps, uint64_t num_tokens, float max_shift, float base_shift,
                          int32_t stretch, float terminal, float *sigmas_out);
/* make_target_positions (patchifier.rs:101-118): [batch, 3, F*H*W, 2] f32
 * pixel/time bounds with the causal fix, into host memory (bit-exact).
 * LTX-2 scale factors are (8, 32, 32).  Host-only. */
int ltx_target_positions(uint32_t frames, uint32_t height, uint32_t width, uint32_t batch, uint32_t scale_t,
                         uint32_t scale_h, uint32_t scale_w, float fps, float *out_host);
/* make_reference_positions (patchifier.rs:131-161) for IC-LoRA reference
 * tokens, into host memory (bit-exact).  Host-only. */
int ltx_reference_positions(uint32_t frames, uint32_t height, uint32_t width, uint32_t batch,
                            uint32_t first_latent_frame, uint32_t scale_t, uint32_t scale_h, uint32_t scale_w,
                            float fps, uint32_t temporal_scale_factor, uint32_t downscale_factor,
                            float *out_host);
/* patchify / unpatchify (patchifier.rs:50-89), patch size 1, on the device:
 * [B, C, F, H, W] <-> [B, F*H*W, C] f32. */
int ltx_patchify(ltx_ctx *ctx, const float *latent_dev, int32_t batch, int32_t channels, int32_t frames,
                 int32_t height, int32_t width, float *tokens_dev);
int ltx_unpatchify(ltx_ctx *ctx, const float *tokens_dev, int32_t batch, int32_t channels, int32_t frames,
                   int32_t height, int32_t width, float *latent_dev);

/* ---- temporal chunks (crates/ltx-chunk) ---------------------------------- */

/* ltx_chunk::plan::Chunk (crates/ltx-chunk/src/plan.rs:24-35): frames
 * [start, end) of the clip, and the frames shared with the previous chunk. */
typedef struct {
    uint32_t start;
    uint32_t end;
    uint32_t real_overlap;
} ltx_chunk;

/* ltx_chunk::plan::plan (plan.rs:56-160): overlapping windows of chunk_len
 * (8k+1) frames, stride chunk_len - overlap, the last one anchored to the
 * clip's end.  Writes at most max_chunks entries and the count to *n_chunks
 * (the count is written even when max_chunks is too small, which returns
 * LTX_ERR_INVALID_ARG).  Errors (LTX_ERR_CHUNK_PLAN) mirror ChunkError:
 * ZeroTotal, ChunkLenNotOnGrid, OverlapNotSmallerThanChunkLen,
 * OverlapNotMultipleOf8, StrideSmallerThanOverlap; ltx_host_last_error()
 * names the variant.  Host-only. */
int ltx_chunk_plan(uint32_t total, uint32_t chunk_len, uint32_t overlap, ltx_chunk *chunks_out,
                   int32_t max_chunks, int32_t *n_chunks);
/* seam_cond_plan (crates/ltx-chunk/src/seam.rs:110-125): the keyframe
 * conditioning chunk n > 0 takes from chunk n-1's output at the seam: one
 * frame at chunk-local index 0 with strength 0.95 (DEFAULT_KEYFRAME_STRENGTH),
 * and overlap - 1 frames left to the blend.  LTX_ERR_CHUNK_PLAN
 * (ZeroOverlapForSeam) when overlap is 0.  Host-only. */
int ltx_seam_cond_plan(uint32_t overlap, uint32_t *chunk_local_idx, float *strength, uint32_t *blend_tail_len);
/* crossfade_weight (crates/ltx-chunk/src/blend.rs:49-56): f32 of the f64
 * smoothstep(offset / overlap_len); 1 when overlap_len is 0.  Host-only. */
float ltx_crossfade_weight(uint32_t offset, uint32_t overlap_len);
/* One seam of Blender::finish_chunk (blend.rs:176-182, 284-298) on the
 * device: for frame i < overlap_frames and every value j of the frame,
 *   w = crossfade_weight(i, overlap_frames),
 *   dst[i][j] = fma(w, incoming[i][j], (1 - w) * outgoing[i][j])   (f32),
 * bit-exact with the reference.  Frames are frame_values contiguous f32 (a
 * pixel frame, or a latent frame of H*W tokens x C channels).  dst may alias
 * incoming or outgoing. */
int ltx_seam_blend(ltx_ctx *ctx, const float *outgoing_dev, const float *incoming_dev, uint32_t overlap_frames,
                   int64_t frame_values, float *dst_dev);
/* The whole clip as the reference's streaming Blender emits it (blend.rs
 * finish_chunk / flush, driven as in ltx-pipeline/src/lib.rs:270-353), on
 * the device: chunk_dev[n] holds chunks[n]'s (end - start) frames; dst_dev
 * receives chunks[n_chunks-1].end frames.  Frames covered by one chunk are
 * copied, seam frames are blended as ltx_seam_blend.  chunk_dev is a host
 * array of device pointers; the plan must be one ltx_chunk_plan produced. */
int ltx_chunk_assemble(ltx_ctx *ctx, const float *const *chunk_dev, const ltx_chunk *chunks, int32_t n_chunks,
                       int64_t frame_values, float *dst_dev);

#ifdef __cplusplus
}
#endif

#endif /* LTX_B200_H */
