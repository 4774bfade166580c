// Internal launchers shared between the kernels and the host-side model code.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "internal.hpp"

namespace ltx {

// dequant_merge.cu
int dequant_merge(ltx_ctx *ctx, cudaStream_t stream, const void *w, int w_dt, int has_scale, float scale, int64_t rows,
                  int64_t cols, const ltx_lora_delta *deltas, int n_deltas, void *dst, int dst_dt);

// gemm.cu (epilogue codes = ltx_epilogue)
struct TpGather;
int gemm_bf16(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const void *W, int64_t ldw, int M, int N,
              int K, int epi, const float *bias, void *out, int64_t ldo, const float *gate, const int *gate_idx,
              int64_t ld_gate, int f16_from_col = 1 << 30, const TpGather *ag = nullptr);
// Sequence-parallel gather of normalised rows over the tensor-parallel ranks:
// a GEMM whose A rows of other ranks' M-blocks arrive from their owners waits
// (in its TMA producer, bounded) for the owner's stamp of that M-block.
struct TpGather {
    const uint32_t *stamp;   // this rank's stamps [n-1][mcap]
    uint32_t epoch;
    int n, me, mcap;
};
// Where a norm kernel of the split model also sends its rows: every rank's
// copy of the normalised rows (at the launch's first row), every rank's
// stamps, and this rank's per-M-block block counters.
struct TpNormPush {
    char *peer_out[kMaxTpPeers];
    uint32_t *peer_stamp[kMaxTpPeers];
    uint32_t *count;
    int n, me, mcap, row0;   // row0: the launch's first row, a multiple of 128
    uint32_t epoch;
};
// Row-split projection of a model split over ranks, the sum over ranks and
// the residual update fused (x = ctx->pm's residual; N = pm.D, a multiple of
// 256): x += (sum_r A_r . W_r^T + bias) * gate[gate_idx[row]] on every rank.
// Every rank of the communicator reaches this point of its stream before any
// goes on (collective; bounded wait).
int tp_peer_barrier(ltx_ctx *ctx, cudaStream_t st);
// bcast: also write the finished rows into every other rank's x (false: each
// rank keeps only its own rows current, the sequence-parallel layout).
int gemm_tp_resid(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const void *W, int64_t ldw, int M, int N,
                  int K, const float *bias, const float *gate, const int *gate_idx, int64_t ld_gate, bool bcast = true);
// A bf16 block appended to an e4m3 GEMM's K loop, accumulated into the same
// TMEM accumulator before the scales: acc += A2[M, k2] . B2[N, k2]^T
// (k2 a multiple of 64; leading dimensions in elements).
struct GemmLowRank {
    const void *a2;
    int64_t lda2;
    const void *b2;
    int64_t ldb2;
    int k2;
};
// e4m3 operands (lda/ldw multiples of 16); acc * a_scale[row] * (w_col_scale
// ? w_col_scale[col] : w_scale) before the epilogue
int gemm_e4m3(ltx_ctx *ctx, cudaStream_t st, const void *A, int64_t lda, const float *a_scale, const void *W,
              int64_t ldw, float w_scale, int M, int N, int K, int epi, const float *bias, void *out, int64_t ldo,
              const float *gate, const int *gate_idx, int64_t ld_gate, int f16_from_col = 1 << 30,
              const GemmLowRank *lr = nullptr, const float *w_col_scale = nullptr);

// attention.cu (head_dim 128)
int attention_fwd(ltx_ctx *ctx, cudaStream_t st, const void *q, int64_t ldq, const void *k, int64_t ldk, const void *v,
                  int64_t ldv, int B, int H, int Tq, int Tk, float scale, void *out, int64_t ldo, bool v_f16);

// dit_kernels.cu
cudaError_t rope_table(cudaStream_t st, int sms, const float *pos, int B, int T, const float *freq, int grid,
                       const float max_pos[3], bool use_mid, bool interleaved, int width, float *cos_out,
                       float *sin_out);
cudaError_t norm_mod(cudaStream_t st, const float *x, int64_t ldx, int rows, int D, float eps, int mode,
                     const float *tab, int tab_coeff, const int *idx, int k_shift, __nv_bfloat16 *out, int64_t ldo);
// norm_mod of `rows` rows (D 4096, 16-byte aligned) that also writes each row
// into every other rank's copy and stamps each finished M-block there.
struct TpNormPush;
cudaError_t norm_mod_push(cudaStream_t st, const float *x, int64_t ldx, int rows, float eps, int mode, const float *tab,
                          int tab_coeff, const int *idx, int k_shift, __nv_bfloat16 *out, int64_t ldo,
                          const TpNormPush &push);
cudaError_t ada_tables(cudaStream_t st, int sms, const float *const *sst_dev, int L, int coeff, const float *mod,
                       const float *sst_out, const float *emb, int U, int D, float *tab, float *otab);
cudaError_t qk_norm_rope(cudaStream_t st, __nv_bfloat16 *buf, int64_t ld, int rows, int D, int H, float eps,
                         const float *gamma, const float *cos_t, const float *sin_t, bool interleaved);
cudaError_t sinusoid(cudaStream_t st, const float *ts, int U, float ts_mult, const float *freq, float *out);
cudaError_t small_linear(cudaStream_t st, const float *x, int U, int K, const float *W, const float *bias, int N,
                         bool silu_in, float *out);
cudaError_t f32_to_bf16(cudaStream_t st, int sms, const float *in, int64_t n, __nv_bfloat16 *out);
cudaError_t ctx_mod(cudaStream_t st, int sms, const float *ctx, int64_t n, int D, const float *pst, __nv_bfloat16 *out);
cudaError_t head_gate(cudaStream_t st, int sms, __nv_bfloat16 *o, int64_t ldo, const float *logits, int64_t ldl,
                      int rows, int H, int d);
cudaError_t attention_generic(cudaStream_t st, const __nv_bfloat16 *q, int64_t ldq, const __nv_bfloat16 *k, int64_t ldk,
                              const __nv_bfloat16 *v, int64_t ldv, int B, int H, int Tq, int Tk, int d, float scale,
                              __nv_bfloat16 *out, int64_t ldo);
// Fused self-attention Q/K RMSNorm(gamma) + split RoPE from the forward's cos/sin
// tables ([tab_rows][D/2], row = token row % tab_rows); returns false (nothing
// launched) when the shape is not the specialised one (D 4096, head dim 128).
bool qk_norm_rope_fused(cudaStream_t st, __nv_bfloat16 *q, __nv_bfloat16 *k, int64_t ld, int rows, int D, float eps,
                        const float *gq, const float *gk, const float *cos_t, const float *sin_t, int tab_rows,
                        cudaError_t *err);
cudaError_t permute_ct(cudaStream_t st, int sms, const float *in, float *out, int B, int C, int64_t T, bool to_tokens);
size_t cfg_scratch_bytes();
// Distinct per-token timesteps on the device: at most kMaxDistinctTs values,
// sorted by bit pattern into ts_u[umax] (padded with 0), idx[row] = the row's
// table; more than umax distinct values set *flag = code.
constexpr int kMaxDistinctTs = 8;
constexpr int kErrTooManyTimesteps = 1001;   // device error code: more distinct timesteps than kMaxDistinctTs
cudaError_t timestep_set(cudaStream_t st, const float *ts, int64_t rows, int umax, float *ts_u, int *idx, int *flag,
                         int code);
// ts[h*T + t] = mask[t] * sigma for h < halves.
cudaError_t mask_timesteps(cudaStream_t st, int sms, const float *mask, float sigma, int T, int halves, float *ts);
// Per-token modulation tables tab[row][k][d] = sst[k][d] + mod[row][k*D+d], idx[row] = row (KD = K*D).
cudaError_t seam_tables(cudaStream_t st, int sms, const float *sst, const float *mod, int64_t rows, int KD, float *tab,
                        int *idx);
// Split RoPE (B, H, T, dh) tables -> one row of H*dh values per token.
cudaError_t pe_rows(cudaStream_t st, int sms, const float *cin, const float *sin_, int B, int H, int T, int dh,
                    float *cout, float *sout);
cudaError_t cfg_euler(cudaStream_t st, int sms, float *x, const float *vc, const float *vu, const float *tok_t,
                      const float *mask, const float *clean, int T, int C, float g, float rescale, bool use_cfg,
                      double *partial, float sigma, float sigma_next);

// Tensor-parallel pieces (tp_kernels.cu): per-row sums of squares of nseg
// segments, the Q/K RMSNorm(gamma)+RoPE applied with all-rank sums, and the
// residual add of summed partial projections.
cudaError_t tp_sumsq_rows(cudaStream_t st, const __nv_bfloat16 *x, int64_t ld, int rows, int cols, int nseg,
                          int64_t seg_stride, float *out);
cudaError_t tp_norm_apply_rope(cudaStream_t st, __nv_bfloat16 *x, int64_t ld, int rows, int cols, int D, int d,
                               int head0, float eps, const float *gamma, const float *ss, const float *cos_t,
                               const float *sin_t, bool interleaved);
cudaError_t tp_resid_add(cudaStream_t st, int sms, float *x, const __nv_bfloat16 *p, int rows, int D,
                         const float *bias, const float *gate, const int *gidx, int64_t ld_gate);

// FP8 operand producers (fp8_kernels.cu): e4m3 rows with per-row scale amax/448.
cudaError_t norm_mod_e4m3(cudaStream_t st, const float *x, int64_t ldx, int rows, int D, float eps, int mode,
                          const float *tab, int tab_coeff, const int *idx, int k_shift, uint8_t *out, int64_t ldo,
                          float *scale);
cudaError_t quantize_rows_e4m3(cudaStream_t st, const __nv_bfloat16 *in, int64_t ldi, int rows, int cols, uint8_t *out,
                               int64_t ldo, float *scale);
cudaError_t bf16_to_f32(cudaStream_t st, int sms, const __nv_bfloat16 *in, int64_t n, float *out);
cudaError_t scale_pad_bf16(cudaStream_t st, int sms, const __nv_bfloat16 *in, int rows, int cols_in, int cols_out,
                           float mul, __nv_bfloat16 *out);

}  // namespace ltx
