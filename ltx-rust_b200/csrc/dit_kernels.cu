// The DiT's memory-bound kernels (K4 norms/modulation, K5 timestep path,
// RoPE tables, head gating) and the sampler update (K6: CFG + rescale +
// post-process + Euler).  Each cites the reference code it replaces.
#include "device_common.cuh"
#include "internal.hpp"
#include "kernels.hpp"

namespace ltx {

static int grid_for(int64_t n, int sms, int per_sm = 8) {
    return (int)std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, (int64_t)sms * per_sm));
}

namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// Block-wide sum over blockDim.x (a multiple of 32, <= 1024) threads, fixed order.
__device__ float block_sum(float v, float *red) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) red[warp] = v;
    __syncthreads();
    float t = 0.f;
    if (warp == 0) {
        t = lane < nw ? red[lane] : 0.f;
        t = warp_sum(t);
        if (lane == 0) red[32] = t;
    }
    __syncthreads();
    return red[32];
}

// ── RoPE tables (rope.rs:46-167) ─────────────────────────────────────────────

// positions [B, 3, T, 2] -> cos/sin [B*T, width]:
//   split:       width = inner/2, entry pad + g*3 + p, pad = inner/2 - 3*grid
//   interleaved: width = inner,   entries pad + 2*(g*3+p) + {0,1}, pad = inner - 6*grid
// with angle = (((s+e)/2)/max_p * 2 - 1) * freq[g] (or s/max_p without the
// mid-point grid), padding entries cos 1 / sin 0.
__global__ void rope_table_kernel(const float *pos, int B, int T, const float *freq, int grid, float mp0, float mp1,
                                  float mp2, int use_mid, int interleaved, int width, float *cos_out, float *sin_out) {
    const int64_t total = (int64_t)B * T * width;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t bt = i / width;
        const int e = (int)(i % width);
        const int b = (int)(bt / T), t = (int)(bt % T);
        const int used = interleaved ? 6 * grid : 3 * grid;
        const int pad = width - used;
        float c = 1.f, s = 0.f;
        if (e >= pad) {
            const int idx = interleaved ? (e - pad) >> 1 : (e - pad);
            const int g = idx / 3, ax = idx % 3;
            const float *pp = pos + (((int64_t)b * 3 + ax) * T + t) * 2;
            const float mp = ax == 0 ? mp0 : (ax == 1 ? mp1 : mp2);
            const float frac = use_mid ? __fdiv_rn(__fdiv_rn(__fadd_rn(pp[0], pp[1]), 2.0f), mp) : __fdiv_rn(pp[0], mp);
            const float fm = __fadd_rn(__fmul_rn(frac, 2.0f), -1.0f);
            const float ang = __fmul_rn(fm, freq[g]);
            sincosf(ang, &s, &c);
        }
        cos_out[i] = c;
        sin_out[i] = s;
    }
}

// ── norms + adaLN modulation (norm.rs:23-53, block.rs:131-132, :150-151, model.rs:237-253) ──

// One block per row.  mode 0: y = x / sqrt(mean(x^2)+eps)
//                     mode 1: y = rms(x) * (1 + scale) + shift
//                     mode 2: y = layer_norm(x) * (1 + scale) + shift
// shift/scale rows come from a modulation table tab[u][k][D] (u = idx[row]).
__global__ void norm_mod_kernel(const float *x, int64_t ldx, int rows, int D, float eps, int mode, const float *tab,
                                int tab_coeff, const int *idx, int k_shift, __nv_bfloat16 *out, int64_t ldo) {
    __shared__ float red[33];
    const int row = blockIdx.x;
    if (row >= rows) return;
    const float *xr = x + (int64_t)row * ldx;
    float mean = 0.f;
    if (mode == 2) {
        float s = 0.f;
        for (int c = threadIdx.x; c < D; c += blockDim.x) s += xr[c];
        mean = block_sum(s, red) / (float)D;
    }
    float ss = 0.f;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        const float v = xr[c] - mean;
        ss += v * v;
    }
    const float denom = sqrtf(block_sum(ss, red) / (float)D + eps);
    const float *shift = nullptr, *scale = nullptr;
    if (mode != 0) {
        const int u = idx ? idx[row] : 0;
        shift = tab + ((int64_t)u * tab_coeff + k_shift) * D;
        scale = shift + D;
    }
    __nv_bfloat16 *o = out + (int64_t)row * ldo;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        float y = (xr[c] - mean) / denom;
        if (mode != 0) y = y * (scale[c] + 1.0f) + shift[c];
        o[c] = __float2bfloat16_rn(y);
    }
}

// Modulation tables for all blocks at once:
//   tab[l][u][k][c] = sst_l[k][c] + mod[u][k*D + c]   (block.rs:164-198)
// and the output head table
//   otab[u][k][c] = sst_out[k][c] + emb[u][c]         (model.rs:237-245)
__global__ void ada_tables_kernel(const float *const *sst, int L, int coeff, const float *mod, const float *sst_out,
                                  const float *emb, int U, int D, float *tab, float *otab) {
    const int64_t per_block = (int64_t)U * coeff * D;
    const int64_t total = per_block * L + (int64_t)U * 2 * D;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        if (i < per_block * L) {
            const int l = (int)(i / per_block);
            const int64_t r = i % per_block;
            const int u = (int)(r / ((int64_t)coeff * D));
            const int64_t kc = r % ((int64_t)coeff * D);
            tab[i] = sst[l][kc] + mod[(int64_t)u * coeff * D + kc];
        } else {
            const int64_t r = i - per_block * L;
            const int u = (int)(r / (2 * D));
            const int64_t kc = r % (2 * D);
            otab[r] = sst_out[kc] + emb[(int64_t)u * D + kc % D];
        }
    }
}

// ── Q/K RMSNorm(gamma) over the full inner dim + split/interleaved RoPE ──────
// (attention.rs:154-160 with Burn RmsNorm, rope.rs:231-257 / :269-293).
// In place on bf16 rows [rows, D] (leading dimension ld).  One block per row.
__global__ void qk_norm_rope_kernel(__nv_bfloat16 *buf, int64_t ld, int rows, int D, int H, float eps,
                                    const float *gamma, const float *cos_t, const float *sin_t, int interleaved) {
    extern __shared__ float row_s[];
    __shared__ float red[33];
    const int row = blockIdx.x;
    if (row >= rows) return;
    __nv_bfloat16 *xr = buf + (int64_t)row * ld;
    float ss = 0.f;
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
        const float v = __bfloat162float(xr[c]);
        row_s[c] = v;
        ss += v * v;
    }
    const float denom = sqrtf(block_sum(ss, red) / (float)D + eps);
    for (int c = threadIdx.x; c < D; c += blockDim.x) row_s[c] = row_s[c] / denom * gamma[c];
    __syncthreads();
    if (!cos_t) {
        for (int c = threadIdx.x; c < D; c += blockDim.x) xr[c] = __float2bfloat16_rn(row_s[c]);
        return;
    }
    if (!interleaved) {
        const int d = D / H, half = d / 2, width = D / 2;
        const float *cr = cos_t + (int64_t)row * width, *sr = sin_t + (int64_t)row * width;
        for (int i = threadIdx.x; i < width; i += blockDim.x) {
            const int h = i / half, j = i % half;
            const float x1 = row_s[h * d + j], x2 = row_s[h * d + half + j];
            const float c = cr[i], s = sr[i];
            xr[h * d + j] = __float2bfloat16_rn(c * x1 - s * x2);
            xr[h * d + half + j] = __float2bfloat16_rn(s * x1 + c * x2);
        }
    } else {
        const float *cr = cos_t + (int64_t)row * D, *sr = sin_t + (int64_t)row * D;
        for (int c = threadIdx.x; c < D; c += blockDim.x) {
            const float rot = (c & 1) ? row_s[c - 1] : -row_s[c + 1];
            xr[c] = __float2bfloat16_rn(row_s[c] * cr[c] + rot * sr[c]);
        }
    }
}

// ── timestep path (adaln.rs:43-142, model.rs:196-206) ────────────────────────

__global__ void sinusoid_kernel(const float *ts, int U, float ts_mult, const float *freq, float *out) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= U * 128) return;
    const int u = i / 128, f = i % 128;
    const float ang = __fmul_rn(__fmul_rn(ts[u], ts_mult), freq[f]);
    float s, c;
    sincosf(ang, &s, &c);
    out[u * 256 + f] = c;
    out[u * 256 + 128 + f] = s;
}

__device__ __forceinline__ float silu(float v) { return v / (1.0f + expf(-v)); }

// out[u][n] = bias[n] + sum_k f(x[u][k]) W[n][k], f = SiLU or identity; f32
// weights and accumulation (the timestep MLP and adaLN projection run on the
// few distinct timesteps only).  One warp per output column, U <= 4 rows per pass.
__global__ void small_linear_kernel(const float *x, int U, int K, const float *W, const float *bias, int N, int silu_in,
                                    float *out) {
    extern __shared__ float xs[];   // [4][K]
    const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
    for (int u0 = 0; u0 < U; u0 += 4) {
        const int nu = min(4, U - u0);
        __syncthreads();
        for (int i = threadIdx.x; i < nu * K; i += blockDim.x) {
            const float v = x[(int64_t)(u0 + i / K) * K + i % K];
            xs[i] = silu_in ? silu(v) : v;
        }
        __syncthreads();
        if (warp < N) {
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const float *w = W + (int64_t)warp * K;
            for (int k = lane; k < K; k += 32) {
                const float wv = w[k];
#pragma unroll
                for (int r = 0; r < 4; ++r)
                    if (r < nu) acc[r] += wv * xs[r * K + k];
            }
#pragma unroll
            for (int r = 0; r < 4; ++r) {
                const float s = warp_sum(acc[r]);
                if (lane == 0 && r < nu) out[(int64_t)(u0 + r) * N + warp] = s + (bias ? bias[warp] : 0.f);
            }
        }
    }
}

// ── small elementwise helpers ────────────────────────────────────────────────

__global__ void f32_to_bf16_kernel(const float *in, int64_t n, __nv_bfloat16 *out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = __float2bfloat16_rn(in[i]);
}

// ctx' = ctx * (1 + pst[1]) + pst[0], bf16 out (block.rs:217-223, cross-attention AdaLN flag path).
__global__ void ctx_mod_kernel(const float *ctx, int64_t n, int D, const float *pst, __nv_bfloat16 *out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int c = (int)(i % D);
        out[i] = __float2bfloat16_rn(ctx[i] * (pst[D + c] + 1.0f) + pst[c]);
    }
}

// out[row][h*d + c] *= 2 * sigmoid(logit[row][h])   (attention.rs:180-189)
__global__ void head_gate_kernel(__nv_bfloat16 *o, int64_t ldo, const float *logits, int64_t ldl, int rows, int H,
                                 int d) {
    const int64_t total = (int64_t)rows * H * d;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
        const int row = (int)(i / (H * d));
        const int hc = (int)(i % (H * d));
        const float g = 2.0f / (1.0f + expf(-logits[(int64_t)row * ldl + hc / d]));
        __nv_bfloat16 *p = o + (int64_t)row * ldo + hc;
        *p = __float2bfloat16_rn(__bfloat162float(*p) * g);
    }
}

// ── generic attention for head dims other than 128 (small configs only) ──────
// One block per (batch, head, query row); scores staged in shared memory.
__global__ void attn_generic_kernel(const __nv_bfloat16 *q, int64_t ldq, const __nv_bfloat16 *k, int64_t ldk,
                                    const __nv_bfloat16 *v, int64_t ldv, int B, int H, int Tq, int Tk, int d,
                                    float scale, __nv_bfloat16 *out, int64_t ldo) {
    extern __shared__ float sm[];   // [d] q row, then [Tk] scores
    __shared__ float red[33];
    const int t = blockIdx.x % Tq, h = (blockIdx.x / Tq) % H, b = blockIdx.x / (Tq * H);
    float *qs = sm, *sc = sm + d;
    const __nv_bfloat16 *qr = q + ((int64_t)b * Tq + t) * ldq + h * d;
    for (int c = threadIdx.x; c < d; c += blockDim.x) qs[c] = __bfloat162float(qr[c]);
    __syncthreads();
    float mx = -INFINITY;
    for (int j = threadIdx.x; j < Tk; j += blockDim.x) {
        const __nv_bfloat16 *kr = k + ((int64_t)b * Tk + j) * ldk + h * d;
        float s = 0.f;
        for (int c = 0; c < d; ++c) s += qs[c] * __bfloat162float(kr[c]);
        s *= scale;
        sc[j] = s;
        mx = fmaxf(mx, s);
    }
    // block max
    for (int o = 16; o; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xFFFFFFFFu, mx, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
    __syncthreads();
    if (threadIdx.x == 0) {
        float m = -INFINITY;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) m = fmaxf(m, red[w]);
        red[32] = m;
    }
    __syncthreads();
    const float m = red[32];
    __syncthreads();
    float sum = 0.f;
    for (int j = threadIdx.x; j < Tk; j += blockDim.x) {
        const float p = expf(sc[j] - m);
        sc[j] = p;
        sum += p;
    }
    const float l = block_sum(sum, red);
    for (int c = threadIdx.x; c < d; c += blockDim.x) {
        float acc = 0.f;
        for (int j = 0; j < Tk; ++j) acc += sc[j] * __bfloat162float(v[((int64_t)b * Tk + j) * ldv + h * d + c]);
        out[((int64_t)b * Tq + t) * ldo + h * d + c] = __float2bfloat16_rn(acc / l);
    }
}

// ── K6: CFG + rescale + post-process + Euler (guidance.rs:149-165, loop_.rs:37-65) ──
//
// x0_c = x - t*v_c, x0_u = x - t*v_u  (velocity -> x0 per token, t = mask*sigma;
//                                      tok_t = null: v_c, v_u are x0 predictions)
// pred = x0_c + (g-1)(x0_c - x0_u);  factor = r*std(x0_c)/std(pred) + (1-r)
// x0   = pred*factor;  x0' = x0*m + clean*(1-m);  x += ((x - x0')/sigma)*(sigma_next - sigma)
// Stats: per-block f64 partial sums (sum, sumsq) of x0_c and pred in a fixed
// order, then one block folds them — deterministic for a given grid.

constexpr int kStatBlocks = 256;

__global__ void cfg_stats_kernel(const float *x, const float *vc, const float *vu, const float *tok_t, int T, int C,
                                 float g, double *partial) {
    __shared__ double red[4][32];
    double s[4] = {0, 0, 0, 0};
    const int64_t n = (int64_t)T * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        float xc, xu;
        if (tok_t) {
            const float t = tok_t[i / C];
            xc = x[i] - t * vc[i];
            xu = x[i] - t * vu[i];
        } else {   // the inputs are x0 predictions already
            xc = vc[i];
            xu = vu[i];
        }
        const float pr = xc + (g - 1.0f) * (xc - xu);
        s[0] += xc;
        s[1] += (double)xc * xc;
        s[2] += pr;
        s[3] += (double)pr * pr;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        double v = s[q];
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
        if (lane == 0) red[q][warp] = v;
    }
    __syncthreads();
    if (threadIdx.x < 4) {
        double v = 0;
        for (int w = 0; w < (int)(blockDim.x >> 5); ++w) v += red[threadIdx.x][w];
        partial[blockIdx.x * 4 + threadIdx.x] = v;
    }
}

__global__ void cfg_euler_apply_kernel(float *x, const float *vc, const float *vu, const float *tok_t, const float *mask,
                                       const float *clean, int T, int C, float g, float rescale, int use_cfg,
                                       const double *partial, int nparts, float sigma, float sigma_next) {
    __shared__ float factor_s;
    if (threadIdx.x == 0) {
        float factor = 1.0f;
        if (use_cfg && fabsf(rescale) >= 1e-6f) {
            double s[4] = {0, 0, 0, 0};
            for (int b = 0; b < nparts; ++b)
                for (int q = 0; q < 4; ++q) s[q] += partial[b * 4 + q];
            const double n = (double)T * C;
            const double mc = s[0] / n, mp = s[2] / n;
            const double vc_ = s[1] / n - mc * mc, vp = s[3] / n - mp * mp;
            const double sc = sqrt(fmax(vc_, 0.0) + 1e-8), sp = sqrt(fmax(vp, 0.0) + 1e-8);
            factor = (float)(rescale * (sc / sp) + (1.0 - rescale));
        }
        factor_s = factor;
    }
    __syncthreads();
    const float factor = factor_s;
    const float dt = sigma_next - sigma;
    const int64_t n = (int64_t)T * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t tok = i / C;
        const float xi = x[i];
        float x0;
        if (tok_t) {
            const float t = tok_t[tok];
            const float xc = xi - t * vc[i];
            x0 = xc;
            if (use_cfg) {
                const float xu = xi - t * vu[i];
                x0 = (xc + (g - 1.0f) * (xc - xu)) * factor;
            }
        } else {   // the inputs are x0 predictions already
            const float xc = vc[i];
            x0 = xc;
            if (use_cfg) {
                const float xu = vu[i];
                x0 = (xc + (g - 1.0f) * (xc - xu)) * factor;
            }
        }
        const float m = mask[tok];
        const float x0a = x0 * m + clean[i] * (1.0f - m);
        const float vel = (xi - x0a) / sigma;
        x[i] = xi + vel * dt;
    }
}

// ── distinct timesteps on the device ────────────────────────────────────────
//
// The adaLN path runs once per distinct timestep value (model.rs:196-206 runs
// it per token, with the same result).  One CTA collects the distinct f32 bit
// patterns of ts[rows] (up to umax), sorts them by bit pattern so the table
// order is deterministic, writes them to ts_u (padded with 0) and each row's
// index to idx.  More than umax distinct values: `flag` gets `code`.
__global__ void __launch_bounds__(1024) timestep_set_kernel(const float *ts, int64_t rows, int umax, float *ts_u,
                                                            int *idx, int *flag, int code) {
    constexpr uint32_t kEmpty = 0xFFFFFFFFu;   // a NaN pattern: stands for "no value"
    __shared__ uint32_t vals[kMaxDistinctTs];
    __shared__ int overflow;
    for (int k = threadIdx.x; k < kMaxDistinctTs; k += blockDim.x) vals[k] = kEmpty;
    if (threadIdx.x == 0) overflow = 0;
    __syncthreads();
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
        const uint32_t b = __float_as_uint(ts[r]);
        bool placed = false;
        for (int k = 0; k < umax && !placed; ++k) {
            uint32_t v = vals[k];
            if (v == kEmpty) v = atomicCAS(&vals[k], kEmpty, b);
            placed = v == kEmpty || v == b;
        }
        if (!placed) overflow = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = 0;
        while (n < umax && vals[n] != kEmpty) ++n;
        for (int i = 1; i < n; ++i)   // insertion sort of at most umax patterns
            for (int j = i; j > 0 && vals[j - 1] > vals[j]; --j) {
                const uint32_t t = vals[j];
                vals[j] = vals[j - 1];
                vals[j - 1] = t;
            }
        for (int k = 0; k < umax; ++k) ts_u[k] = k < n ? __uint_as_float(vals[k]) : 0.0f;
        if (overflow && flag) atomicExch(flag, code);
    }
    __syncthreads();
    for (int64_t r = threadIdx.x; r < rows; r += blockDim.x) {
        const uint32_t b = __float_as_uint(ts[r]);
        int k = 0;
        while (k + 1 < umax && vals[k] != b) ++k;
        idx[r] = k;
    }
}

// Per-token timesteps of a denoise step, t = mask * sigma (guidance.rs:114),
// for each of the `halves` batch rows of the CFG batch.
__global__ void mask_timesteps_kernel(const float *mask, float sigma, int T, int halves, float *ts) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)T * halves;
         i += (int64_t)gridDim.x * blockDim.x)
        ts[i] = mask[i % T] * sigma;
}

// ── the block seam: TransformerBlock::forward's own inputs ────────────────────
//
// tab[row][k][d] = sst[k][d] + mod[row][k*D + d] (ada_values, block.rs:164-198,
// per token) and idx[row] = row, so the norm and GEMM-epilogue kernels read
// per-token modulation the way they read the per-timestep tables.
__global__ void seam_tables_kernel(const float *sst, const float *mod, int64_t rows, int KD, float *tab, int *idx) {
    const int64_t n = rows * KD;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        tab[i] = sst[i % KD] + mod[i];
        if (i % KD == 0) idx[i / KD] = (int)(i / KD);
    }
}

// Split RoPE tables from the reference's layout (B, H, T, dh) (split_freqs_cis,
// rope.rs:118-167) to one row per token: out[(b*T + t)*H*dh + h*dh + i].
__global__ void pe_rows_kernel(const float *cin, const float *sin_, int B, int H, int T, int dh, float *cout,
                               float *sout) {
    const int64_t n = (int64_t)B * H * T * dh;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int e = (int)(i % dh);
        const int64_t r = i / dh;
        const int t = (int)(r % T), h = (int)((r / T) % H), b = (int)(r / ((int64_t)T * H));
        const int64_t o = ((int64_t)b * T + t) * H * dh + (int64_t)h * dh + e;
        cout[o] = cin[i];
        sout[o] = sin_[i];
    }
}

// patchify (patchifier.rs:50-60): [B, C, T] -> [B, T, C], T = F*H*W (patch size 1);
// unpatchify the inverse.  Pure index permutation (bit-exact).
__global__ void permute_ct_kernel(const float *in, float *out, int B, int C, int64_t T, int to_tokens) {
    const int64_t n = (int64_t)B * C * T;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t b = i / ((int64_t)C * T), r = i % ((int64_t)C * T);
        if (to_tokens) {   // i indexes the token layout [b][t][c]
            const int64_t t = r / C, c = r % C;
            out[i] = in[(b * C + c) * T + t];
        } else {           // i indexes the latent layout [b][c][t]
            const int64_t c = r / T, t = r % T;
            out[i] = in[(b * T + t) * C + c];
        }
    }
}

// ── warp-per-row variants for the production shapes (D a multiple of 128) ───

__device__ __forceinline__ float warp_sum_all(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xFFFFFFFFu, v, o);
    return v;
}

// norm_mod for D = 4096 with each row split over SPLIT warps (lane l of part w
// owns float4 columns w*D/SPLIT + l*4 + 128*i): the row stays in registers
// with a per-thread state small enough for 2 blocks (16 warps) per SM.  The partial sums
// meet in shared memory.  Same modes and results as norm_mod_kernel.
// PUSH (a model split over ranks, sequence-parallel norms): every row also
// goes into every other rank's copy of `out`, and the last block of each
// 128-row M-block stamps that M-block on every other rank.
template <int SPLIT, bool PUSH = false>
__global__ void __launch_bounds__(256) norm_mod_split_kernel(const float *x, int64_t ldx, int rows, float eps, int mode,
                                                             const float *tab, int tab_coeff, const int *idx,
                                                             int k_shift, __nv_bfloat16 *out, int64_t ldo,
                                                             TpNormPush push = TpNormPush{}) {
    constexpr int D = 4096, NV = D / 128 / SPLIT, RPB = 8 / SPLIT;   // float4 per lane, rows per block
    __shared__ float part[2][8];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rib = warp / SPLIT, piece = warp % SPLIT;
    const int row = blockIdx.x * RPB + rib;
    const bool live = row < rows;
    const int col0 = piece * (D / SPLIT);
    float4 v[NV];
    if (live) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + (int64_t)row * ldx + col0);
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = __ldcs(xr + lane + 32 * i);
    } else {
#pragma unroll
        for (int i = 0; i < NV; ++i) v[i] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    float mean = 0.f;
    if (mode == 2) {
        float s = 0.f;
#pragma unroll
        for (int i = 0; i < NV; ++i) s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
        s = warp_sum_all(s);
        if (lane == 0) part[0][warp] = s;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int q = 0; q < SPLIT; ++q) tot += part[0][rib * SPLIT + q];
        mean = tot / (float)D;
    }
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        v[i].x -= mean; v[i].y -= mean; v[i].z -= mean; v[i].w -= mean;
        ss += v[i].x * v[i].x + v[i].y * v[i].y + v[i].z * v[i].z + v[i].w * v[i].w;
    }
    ss = warp_sum_all(ss);
    if (lane == 0) part[1][warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int q = 0; q < SPLIT; ++q) tot += part[1][rib * SPLIT + q];
    if (!PUSH && !live) return;
    const float denom = sqrtf(tot / (float)D + eps);
    const float4 *sh = nullptr, *sc = nullptr;
    if (mode != 0 && live) {
        const int u = idx ? idx[row] : 0;
        const float *shift = tab + ((int64_t)u * tab_coeff + k_shift) * D + col0;
        sh = reinterpret_cast<const float4 *>(shift);
        sc = reinterpret_cast<const float4 *>(shift + D);
    }
    uint2 *o = reinterpret_cast<uint2 *>(out + (int64_t)row * ldo + col0);
#pragma unroll
    for (int i = 0; i < NV; ++i) {
        if (!live) break;   // PUSH only (a dead row's block still reaches the report below)
        float a = v[i].x / denom, b = v[i].y / denom, c = v[i].z / denom, d = v[i].w / denom;
        if (mode != 0) {
            const float4 s4 = __ldg(sc + lane + 32 * i), h4 = __ldg(sh + lane + 32 * i);
            a = a * (s4.x + 1.0f) + h4.x;
            b = b * (s4.y + 1.0f) + h4.y;
            c = c * (s4.z + 1.0f) + h4.z;
            d = d * (s4.w + 1.0f) + h4.w;
        }
        __nv_bfloat162 lo = __floats2bfloat162_rn(a, b), hi = __floats2bfloat162_rn(c, d);
        const uint2 val = make_uint2(*reinterpret_cast<uint32_t *>(&lo), *reinterpret_cast<uint32_t *>(&hi));
        o[lane + 32 * i] = val;
        if constexpr (PUSH) {
            for (int q = 0; q < push.n; ++q)
                if (q != push.me)
                    reinterpret_cast<uint2 *>(reinterpret_cast<__nv_bfloat16 *>(push.peer_out[q]) + (int64_t)row * ldo +
                                              col0)[lane + 32 * i] = val;
        }
    }
    if constexpr (PUSH) {
        // Rows of one 128-row M-block: the launch's rows start at a multiple
        // of 128 and a block holds RPB consecutive rows, so no block spans two.
        __threadfence_system();   // this thread's pushes, before the block reports
        __syncthreads();
        if (threadIdx.x == 0) {
            const int r_first = blockIdx.x * RPB;
            const int mb = (push.row0 + r_first) / 128;
            const int in_mb = min(128, push.row0 + rows - mb * 128);
            const unsigned blocks_in_mb = (unsigned)((in_mb + RPB - 1) / RPB);
            if (atomicAdd(push.count + mb, 1u) + 1 == blocks_in_mb) {
                atomicExch(push.count + mb, 0u);
                __threadfence_system();
                for (int q = 0; q < push.n; ++q)
                    if (q != push.me)
                        st_release_sys(push.peer_stamp[q] + (int64_t)(push.me < q ? push.me : push.me - 1) * push.mcap + mb,
                                       push.epoch);
            }
        }
    }
}

// RMSNorm(gamma) over a bf16 row in place (no RoPE), warp per row; lane l owns
// 8-element groups l*8 + 256*i, i < NG (NG = D/256).
template <int NG>
__global__ void __launch_bounds__(256) rmsnorm_gamma_warp_kernel(__nv_bfloat16 *buf, int64_t ld, int rows, float eps,
                                                                 const float *gamma) {
    constexpr int D = NG * 256;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    uint4 *xr = reinterpret_cast<uint4 *>(buf + (int64_t)row * ld);
    float f[NG][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        const uint4 u = xr[lane + 32 * i];
        const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float2 t = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&w[e]));
            f[i][2 * e] = t.x;
            f[i][2 * e + 1] = t.y;
            ss += t.x * t.x + t.y * t.y;
        }
    }
    const float denom = sqrtf(warp_sum_all(ss) / (float)D + eps);
#pragma unroll
    for (int i = 0; i < NG; ++i) {
        const float4 *g4 = reinterpret_cast<const float4 *>(gamma + (lane + 32 * i) * 8);
        const float4 ga = __ldg(g4), gb = __ldg(g4 + 1);
        const float g[8] = {ga.x, ga.y, ga.z, ga.w, gb.x, gb.y, gb.z, gb.w};
        uint32_t w[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            __nv_bfloat162 h = __floats2bfloat162_rn(f[i][2 * e] / denom * g[2 * e], f[i][2 * e + 1] / denom * g[2 * e + 1]);
            w[e] = *reinterpret_cast<uint32_t *>(&h);
        }
        xr[lane + 32 * i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

// Self-attention Q and K of one token, in place: RMSNorm(gamma) over the full
// inner dim for each, then split RoPE with cos/sin read from the forward's
// tables ([table rows][D/2], built once per forward by rope_table_kernel; row
// `row % tab_rows`, so CFG rows that share their positions share one table
// row).  Head dim 128, H = D/128 heads, warp per token; lane l owns pairs
// j = 2l, 2l+1 of every head (columns h*128 + {2l, 2l+1} and
// h*128 + 64 + {2l, 2l+1}), i.e. table entries h*64 + 2l, 2l+1.
template <int H>
__global__ void __launch_bounds__(256) qk_norm_rope_fused_kernel(__nv_bfloat16 *q, __nv_bfloat16 *k, int64_t ld,
                                                                 int rows, float eps, const float *gq, const float *gk,
                                                                 const float *cos_t, const float *sin_t, int tab_rows) {
    constexpr int D = H * 128;
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    uint32_t *qr = reinterpret_cast<uint32_t *>(q + (int64_t)row * ld);
    uint32_t *kr = reinterpret_cast<uint32_t *>(k + (int64_t)row * ld);
    // Phase 1 streams the row for the two sums of squares; phase 2 re-reads it
    // (L1/L2-resident) to normalise, rotate and store.
    float sq = 0.f, sk = 0.f;
#pragma unroll 8
    for (int w = lane; w < D / 2; w += 32) {
        const float2 a = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qr[w]));
        const float2 c = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[w]));
        sq += a.x * a.x + a.y * a.y;
        sk += c.x * c.x + c.y * c.y;
    }
    const float dq = sqrtf(warp_sum_all(sq) / (float)D + eps);
    const float dk = sqrtf(warp_sum_all(sk) / (float)D + eps);
    const int64_t trow = (int64_t)(row % tab_rows) * (D / 2);
    const float2 *ct = reinterpret_cast<const float2 *>(cos_t + trow);
    const float2 *stb = reinterpret_cast<const float2 *>(sin_t + trow);
#pragma unroll 4
    for (int h = 0; h < H; ++h) {
        const float2 qa = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qr[h * 64 + lane]));
        const float2 qb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&qr[h * 64 + 32 + lane]));
        const float2 ka = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[h * 64 + lane]));
        const float2 kb = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162 *>(&kr[h * 64 + 32 + lane]));
        const float2 c2 = __ldg(ct + h * 32 + lane), s2 = __ldg(stb + h * 32 + lane);
        const float c[2] = {c2.x, c2.y}, s[2] = {s2.x, s2.y};
        const int col = h * 128 + 2 * lane;
        const float q1x = qa.x / dq * __ldg(gq + col), q1y = qa.y / dq * __ldg(gq + col + 1);
        const float q2x = qb.x / dq * __ldg(gq + col + 64), q2y = qb.y / dq * __ldg(gq + col + 65);
        const float k1x = ka.x / dk * __ldg(gk + col), k1y = ka.y / dk * __ldg(gk + col + 1);
        const float k2x = kb.x / dk * __ldg(gk + col + 64), k2y = kb.y / dk * __ldg(gk + col + 65);
        __nv_bfloat162 o;
        o = __floats2bfloat162_rn(c[0] * q1x - s[0] * q2x, c[1] * q1y - s[1] * q2y);
        qr[h * 64 + lane] = *reinterpret_cast<uint32_t *>(&o);
        o = __floats2bfloat162_rn(s[0] * q1x + c[0] * q2x, s[1] * q1y + c[1] * q2y);
        qr[h * 64 + 32 + lane] = *reinterpret_cast<uint32_t *>(&o);
        o = __floats2bfloat162_rn(c[0] * k1x - s[0] * k2x, c[1] * k1y - s[1] * k2y);
        kr[h * 64 + lane] = *reinterpret_cast<uint32_t *>(&o);
        o = __floats2bfloat162_rn(s[0] * k1x + c[0] * k2x, s[1] * k1y + c[1] * k2y);
        kr[h * 64 + 32 + lane] = *reinterpret_cast<uint32_t *>(&o);
    }
}

}  // namespace

bool qk_norm_rope_fused(cudaStream_t st, __nv_bfloat16 *q, __nv_bfloat16 *k, int64_t ld, int rows, int D, float eps,
                        const float *gq, const float *gk, const float *cos_t, const float *sin_t, int tab_rows,
                        cudaError_t *err) {
    if (D != 4096 || (ld % 2) || ((uintptr_t)q & 3) || ((uintptr_t)k & 3) || ((uintptr_t)cos_t & 7) ||
        ((uintptr_t)sin_t & 7) || tab_rows <= 0)
        return false;
    qk_norm_rope_fused_kernel<32><<<(rows + 7) / 8, 256, 0, st>>>(q, k, ld, rows, eps, gq, gk, cos_t, sin_t, tab_rows);
    *err = cudaGetLastError();
    return true;
}

cudaError_t permute_ct(cudaStream_t st, int sms, const float *in, float *out, int B, int C, int64_t T, bool to_tokens) {
    permute_ct_kernel<<<grid_for((int64_t)B * C * T, sms), 256, 0, st>>>(in, out, B, C, T, to_tokens);
    return cudaGetLastError();
}

// ── launchers (kernels.hpp) ──────────────────────────────────────────────────


cudaError_t rope_table(cudaStream_t st, int sms, const float *pos, int B, int T, const float *freq, int grid,
                       const float max_pos[3], bool use_mid, bool interleaved, int width, float *cos_out,
                       float *sin_out) {
    rope_table_kernel<<<grid_for((int64_t)B * T * width, sms), 256, 0, st>>>(
        pos, B, T, freq, grid, max_pos[0], max_pos[1], max_pos[2], use_mid, interleaved, width, cos_out, sin_out);
    return cudaGetLastError();
}

cudaError_t norm_mod(cudaStream_t st, const float *x, int64_t ldx, int rows, int D, float eps, int mode,
                     const float *tab, int tab_coeff, const int *idx, int k_shift, __nv_bfloat16 *out, int64_t ldo) {
    if (rows <= 0) return cudaSuccess;
    const bool vec = ldx % 4 == 0 && ldo % 4 == 0 && ((uintptr_t)x & 15) == 0 && ((uintptr_t)out & 7) == 0 &&
                     (!tab || ((uintptr_t)tab & 15) == 0);
    if (vec && D == 4096) {
        // two warps per row, 4 rows per 256-thread block
        norm_mod_split_kernel<2><<<(rows + 3) / 4, 256, 0, st>>>(x, ldx, rows, eps, mode, tab, tab_coeff, idx, k_shift,
                                                                  out, ldo);
        return cudaGetLastError();
    }
    norm_mod_kernel<<<rows, 256, 0, st>>>(x, ldx, rows, D, eps, mode, tab, tab_coeff, idx, k_shift, out, ldo);
    return cudaGetLastError();
}

cudaError_t norm_mod_push(cudaStream_t st, const float *x, int64_t ldx, int rows, float eps, int mode, const float *tab,
                          int tab_coeff, const int *idx, int k_shift, __nv_bfloat16 *out, int64_t ldo,
                          const TpNormPush &push) {
    if (rows <= 0) return cudaSuccess;
    if (push.row0 % 128 || ldx % 4 || ldo % 4 || ((uintptr_t)x & 15) || ((uintptr_t)out & 7) ||
        (tab && ((uintptr_t)tab & 15)))
        return cudaErrorInvalidValue;
    norm_mod_split_kernel<2, true><<<(rows + 3) / 4, 256, 0, st>>>(x, ldx, rows, eps, mode, tab, tab_coeff, idx, k_shift,
                                                                    out, ldo, push);
    return cudaGetLastError();
}

cudaError_t ada_tables(cudaStream_t st, int sms, const float *const *sst_dev, int L, int coeff, const float *mod,
                       const float *sst_out, const float *emb, int U, int D, float *tab, float *otab) {
    const int64_t total = (int64_t)L * U * coeff * D + (int64_t)U * 2 * D;
    ada_tables_kernel<<<grid_for(total, sms), 256, 0, st>>>(sst_dev, L, coeff, mod, sst_out, emb, U, D, tab, otab);
    return cudaGetLastError();
}

cudaError_t qk_norm_rope(cudaStream_t st, __nv_bfloat16 *buf, int64_t ld, int rows, int D, int H, float eps,
                         const float *gamma, const float *cos_t, const float *sin_t, bool interleaved) {
    if (rows <= 0) return cudaSuccess;
    if (!cos_t && D == 4096 && ld % 8 == 0 && ((uintptr_t)buf & 15) == 0 && ((uintptr_t)gamma & 15) == 0) {
        rmsnorm_gamma_warp_kernel<16><<<(rows + 7) / 8, 256, 0, st>>>(buf, ld, rows, eps, gamma);
        return cudaGetLastError();
    }
    const size_t smem = (size_t)D * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(qk_norm_rope_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    qk_norm_rope_kernel<<<rows, 256, smem, st>>>(buf, ld, rows, D, H, eps, gamma, cos_t, sin_t, interleaved);
    return cudaGetLastError();
}

cudaError_t sinusoid(cudaStream_t st, const float *ts, int U, float ts_mult, const float *freq, float *out) {
    sinusoid_kernel<<<(U * 128 + 127) / 128, 128, 0, st>>>(ts, U, ts_mult, freq, out);
    return cudaGetLastError();
}

cudaError_t small_linear(cudaStream_t st, const float *x, int U, int K, const float *W, const float *bias, int N,
                         bool silu_in, float *out) {
    const size_t smem = (size_t)4 * K * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(small_linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    const int warps_per_block = 8;
    small_linear_kernel<<<(N + warps_per_block - 1) / warps_per_block, warps_per_block * 32, smem, st>>>(
        x, U, K, W, bias, N, silu_in, out);
    return cudaGetLastError();
}

cudaError_t f32_to_bf16(cudaStream_t st, int sms, const float *in, int64_t n, __nv_bfloat16 *out) {
    f32_to_bf16_kernel<<<grid_for(n, sms), 256, 0, st>>>(in, n, out);
    return cudaGetLastError();
}

cudaError_t ctx_mod(cudaStream_t st, int sms, const float *ctx, int64_t n, int D, const float *pst, __nv_bfloat16 *out) {
    ctx_mod_kernel<<<grid_for(n, sms), 256, 0, st>>>(ctx, n, D, pst, out);
    return cudaGetLastError();
}

cudaError_t head_gate(cudaStream_t st, int sms, __nv_bfloat16 *o, int64_t ldo, const float *logits, int64_t ldl,
                      int rows, int H, int d) {
    head_gate_kernel<<<grid_for((int64_t)rows * H * d, sms), 256, 0, st>>>(o, ldo, logits, ldl, rows, H, d);
    return cudaGetLastError();
}

cudaError_t attention_generic(cudaStream_t st, const __nv_bfloat16 *q, int64_t ldq, const __nv_bfloat16 *k, int64_t ldk,
                              const __nv_bfloat16 *v, int64_t ldv, int B, int H, int Tq, int Tk, int d, float scale,
                              __nv_bfloat16 *out, int64_t ldo) {
    const size_t smem = (size_t)(d + Tk) * sizeof(float);
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(attn_generic_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    attn_generic_kernel<<<B * H * Tq, 128, smem, st>>>(q, ldq, k, ldk, v, ldv, B, H, Tq, Tk, d, scale, out, ldo);
    return cudaGetLastError();
}

size_t cfg_scratch_bytes() { return (size_t)kStatBlocks * 4 * sizeof(double); }

cudaError_t timestep_set(cudaStream_t st, const float *ts, int64_t rows, int umax, float *ts_u, int *idx, int *flag,
                         int code) {
    if (umax < 1 || umax > kMaxDistinctTs) return cudaErrorInvalidValue;
    timestep_set_kernel<<<1, 1024, 0, st>>>(ts, rows, umax, ts_u, idx, flag, code);
    return cudaGetLastError();
}

cudaError_t mask_timesteps(cudaStream_t st, int sms, const float *mask, float sigma, int T, int halves, float *ts) {
    mask_timesteps_kernel<<<grid_for((int64_t)T * halves, sms), 256, 0, st>>>(mask, sigma, T, halves, ts);
    return cudaGetLastError();
}

cudaError_t seam_tables(cudaStream_t st, int sms, const float *sst, const float *mod, int64_t rows, int KD, float *tab,
                        int *idx) {
    seam_tables_kernel<<<grid_for(rows * KD, sms), 256, 0, st>>>(sst, mod, rows, KD, tab, idx);
    return cudaGetLastError();
}

cudaError_t pe_rows(cudaStream_t st, int sms, const float *cin, const float *sin_, int B, int H, int T, int dh,
                    float *cout, float *sout) {
    pe_rows_kernel<<<grid_for((int64_t)B * H * T * dh, sms), 256, 0, st>>>(cin, sin_, B, H, T, dh, cout, sout);
    return cudaGetLastError();
}

cudaError_t cfg_euler(cudaStream_t st, int sms, float *x, const float *vc, const float *vu, const float *tok_t,
                      const float *mask, const float *clean, int T, int C, float g, float rescale, bool use_cfg,
                      double *partial, float sigma, float sigma_next) {
    if (use_cfg) {
        cfg_stats_kernel<<<kStatBlocks, 256, 0, st>>>(x, vc, vu, tok_t, T, C, g, partial);
        cudaError_t e = cudaGetLastError();
        if (e != cudaSuccess) return e;
    }
    // The apply kernel folds the partials in every block (256 x 4 doubles, cheap) before updating.
    cfg_euler_apply_kernel<<<grid_for((int64_t)T * C, sms, 4), 256, 0, st>>>(
        x, vc, vu, tok_t, mask, clean, T, C, g, rescale, use_cfg, partial, kStatBlocks, sigma, sigma_next);
    return cudaGetLastError();
}

}  // namespace ltx

extern "C" int ltx_patchify(ltx_ctx *ctx, const float *latent_dev, int32_t batch, int32_t channels, int32_t frames,
                            int32_t height, int32_t width, float *tokens_dev) {
    if (!ctx || batch < 0 || channels < 0 || frames < 0 || height < 0 || width < 0)
        return ctx ? ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_patchify: bad arguments") : LTX_ERR_INVALID_ARG;
    if ((int64_t)batch * channels * frames * height * width == 0) return LTX_OK;   // nothing to move
    if (!latent_dev || !tokens_dev) return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_patchify: null pointer");
    cudaError_t e = ltx::permute_ct(ctx->stream, ctx->sm_count, latent_dev, tokens_dev, batch, channels,
                                    (int64_t)frames * height * width, true);
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_patchify");
}

extern "C" int ltx_unpatchify(ltx_ctx *ctx, const float *tokens_dev, int32_t batch, int32_t channels, int32_t frames,
                              int32_t height, int32_t width, float *latent_dev) {
    if (!ctx || batch < 0 || channels < 0 || frames < 0 || height < 0 || width < 0)
        return ctx ? ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_unpatchify: bad arguments") : LTX_ERR_INVALID_ARG;
    if ((int64_t)batch * channels * frames * height * width == 0) return LTX_OK;   // nothing to move
    if (!latent_dev || !tokens_dev) return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_unpatchify: null pointer");
    cudaError_t e = ltx::permute_ct(ctx->stream, ctx->sm_count, tokens_dev, latent_dev, batch, channels,
                                    (int64_t)frames * height * width, false);
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_unpatchify");
}

// ImageKeyframeCondition::apply_to (crates/ltx-sampler/src/conditioning.rs:
// 127-205): per value, clean*keep + img*frame, and per token mask*keep +
// frame*(1-strength), each Burn op one f32 rounding (keep = 1 - frame).
namespace {
__global__ void apply_keyframe_kernel(float *clean, float *mask, int64_t tokens, int C, const float *image,
                                      int64_t start, int64_t tpf, float one_minus_s) {
    const int64_t n = tokens * C;
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t t = i / C;
        const int c = (int)(i % C);
        const bool in = t >= start && t < start + tpf;
        const float frame = in ? 1.0f : 0.0f, keep = in ? 0.0f : 1.0f;
        const float img = in ? image[(int64_t)c * tpf + (t - start)] : 0.0f;   // patchify of [C, 1, H, W]
        clean[i] = __fadd_rn(__fmul_rn(clean[i], keep), __fmul_rn(img, frame));
        if (c == 0) mask[t] = __fadd_rn(__fmul_rn(mask[t], keep), __fmul_rn(frame, one_minus_s));
    }
}
}  // namespace

extern "C" int ltx_apply_keyframe(ltx_ctx *ctx, float *clean_dev, float *mask_dev, int32_t tokens, int32_t channels,
                                  const float *image_dev, int32_t latent_frame_index, int32_t tokens_per_frame,
                                  float strength) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!(strength >= 0.0f && strength <= 1.0f))
        return ltx::fail(ctx, LTX_ERR_STRENGTH, "InvalidStrength: keyframe strength %g outside [0, 1]", (double)strength);
    if (!clean_dev || !mask_dev || !image_dev || tokens < 0 || channels <= 0 || latent_frame_index < 0 ||
        tokens_per_frame <= 0)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_apply_keyframe: bad arguments");
    const int64_t start = (int64_t)latent_frame_index * tokens_per_frame;
    if (start + tokens_per_frame > tokens)
        return ltx::fail(ctx, LTX_ERR_SHAPE, "image keyframe index exceeds latent frame count");
    const int64_t n = (int64_t)tokens * channels;
    apply_keyframe_kernel<<<ltx::grid_for(n, ctx->sm_count), 256, 0, ctx->stream>>>(
        clean_dev, mask_dev, tokens, channels, image_dev, start, tokens_per_frame, 1.0f - strength);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_apply_keyframe");
}

// GaussianNoiser::apply_with_noise (crates/ltx-sampler/src/noiser.rs:91-106):
// lerp(latent, noise, s) then lerp(clean, noised, mask), each Burn op one f32
// rounding (mul_scalar, add, ones - mask, mul, add), bit-exact.
namespace {
__global__ void apply_noise_kernel(float *latent, const float *noise, const float *clean, const float *mask,
                                   int64_t n, int C, float s, float one_minus_s) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float m = mask[i / C];
        const float noised = __fadd_rn(__fmul_rn(latent[i], one_minus_s), __fmul_rn(noise[i], s));
        latent[i] = __fadd_rn(__fmul_rn(clean[i], __fsub_rn(1.0f, m)), __fmul_rn(noised, m));
    }
}
}  // namespace

extern "C" int ltx_apply_noise(ltx_ctx *ctx, float *latent_dev, const float *noise_dev, const float *clean_dev,
                               const float *mask_dev, int32_t tokens, int32_t channels, float noise_scale) {
    if (!ctx) return LTX_ERR_INVALID_ARG;
    if (!latent_dev || !noise_dev || !clean_dev || !mask_dev || tokens < 0 || channels <= 0)
        return ltx::fail(ctx, LTX_ERR_INVALID_ARG, "ltx_apply_noise: bad arguments");
    const int64_t n = (int64_t)tokens * channels;
    if (n == 0) return LTX_OK;
    apply_noise_kernel<<<ltx::grid_for(n, ctx->sm_count), 256, 0, ctx->stream>>>(latent_dev, noise_dev, clean_dev, mask_dev,
                                                                            n, channels, noise_scale,
                                                                            1.0f - noise_scale);
    cudaError_t e = cudaGetLastError();
    return e == cudaSuccess ? LTX_OK : ltx::cuda_fail(ctx, e, "ltx_apply_noise");
}
